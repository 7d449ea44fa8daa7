"""af_dense_forward_static (parent pass on a file-scope device scratch array) against af_dense_forward.

Two calls in a row of the static entry point must each reproduce the
workspace entry point bit for bit (layer inputs, Q/K/V, logits, self-gate
masks), allocate no device memory (the free
memory the driver reports and torch's allocator are unchanged across the
second call), and sizes whose scratch exceeds the array must be refused with
AF_ERR_CAPACITY before anything is launched. The logit row sums are the one
output compared with a tolerance (1e-5 of the row's absolute logit sum): the
LM-head epilogue adds its per-tile partial sums with fp32 atomics, so their
last bits follow completion order in either entry point.
"""

from __future__ import annotations

import ctypes as C

import pytest
import torch

from actfold_b200 import _lib
from actfold_b200 import workloads as W

pytestmark = pytest.mark.gpu

STATIC_BYTES = 32 << 20  # AF_DENSE_STATIC_WORKSPACE_BYTES


def _outputs(model, T):
    d = model.dims
    dev = model.device
    return dict(
        layer_in=torch.full((d.n_layers + 1, T, d.hidden), 7.0, dtype=torch.bfloat16, device=dev),
        qkv=torch.full((d.n_layers, T, d.q_dim + 2 * d.kv_dim), 7.0, dtype=torch.bfloat16, device=dev),
        logits=torch.full((T, d.vocab), 7.0, dtype=torch.bfloat16, device=dev),
        self_stable=torch.full((d.n_layers, T), 9, dtype=torch.uint8, device=dev),
        row_sums=torch.full((T,), 7.0, dtype=torch.float32, device=dev),
        status=torch.zeros(1, dtype=torch.int32, device=dev),
    )


def _call_static(model, tokens, tau, o):
    from actfold_b200.llada import _bind_late

    lib = _bind_late()
    fn = lib.af_dense_forward_static
    fn.restype, fn.argtypes = _lib.SIGNATURES["af_dense_forward_static"]
    with torch.cuda.device(model.device):
        return fn(C.byref(model._cmodel), tokens.data_ptr(), tokens.numel(), float(tau), o["layer_in"].data_ptr(),
                  o["qkv"].data_ptr(), o["logits"].data_ptr(), o["self_stable"].data_ptr(), o["row_sums"].data_ptr(),
                  o["status"].data_ptr(), _lib.stream_ptr(model.device))


def _same(a, b):
    return torch.equal(a.view(torch.uint8) if a.dtype == torch.bfloat16 else a,
                       b.view(torch.uint8) if b.dtype == torch.bfloat16 else b)


@pytest.mark.parametrize("dims,T", [(W.LLADA_TINY, 128), (W.DREAM_TINY, 200), (W.LLADA_TINY, 1024)])
def test_static_matches_workspace_entry_point(dims, T):
    from actfold_b200.llada import LLaDAModel

    model = LLaDAModel.random(dims, seed=11, device="cuda", std=0.05, max_pos=T)
    g = torch.Generator(device="cpu").manual_seed(T)
    tokens = torch.randint(0, dims.vocab, (T,), generator=g, dtype=torch.int64).cuda()
    ref = model.parent_pass(tokens, tau=0.95)
    torch.cuda.synchronize()

    outs = [_outputs(model, T), _outputs(model, T)]
    st = _call_static(model, tokens, 0.95, outs[0])
    _lib.check(st, "af_dense_forward_static")
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    alloc0 = torch.cuda.memory_allocated()
    st = _call_static(model, tokens, 0.95, outs[1])
    _lib.check(st, "af_dense_forward_static")
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    assert torch.cuda.memory_allocated() == alloc0

    for o in outs:
        assert int(o["status"].item()) == 0
        assert _same(o["layer_in"], ref.layer_in)
        assert _same(o["qkv"], ref.qkv)
        assert _same(o["logits"], ref.logits)
        assert torch.equal(o["self_stable"], ref.self_stable)
        bound = 1e-5 * ref.logits.float().abs().sum(-1) + 1e-6
        assert bool(((o["row_sums"] - ref.row_sums).abs() <= bound).all())


def test_static_rejects_sizes_beyond_the_array():
    from actfold_b200.llada import LLaDAModel, _Dims

    dims = W.LLADA_TINY
    model = LLaDAModel.random(dims, seed=3, device="cuda", std=0.05, max_pos=64)
    lib = _lib.load()
    nb = C.c_int64()
    lib.af_dense_workspace_bytes.restype, lib.af_dense_workspace_bytes.argtypes = _lib.SIGNATURES["af_dense_workspace_bytes"]
    T = 64
    while True:
        _lib.check(lib.af_dense_workspace_bytes(C.byref(model._cdims), T, C.byref(nb)))
        if nb.value > STATIC_BYTES:
            break
        T *= 2
    assert isinstance(model._cdims, _Dims)
    tokens = torch.zeros(T, dtype=torch.int64, device="cuda")
    o = _outputs(model, T)
    st = _call_static(model, tokens, 0.95, o)
    assert st == 2  # AF_ERR_CAPACITY
    msg = _lib.load().af_last_error_string().decode()
    assert "static limit" in msg
    torch.cuda.synchronize()
    assert float(o["row_sums"][0]) == 7.0  # nothing launched
