"""Attention kernel against a plain PyTorch fp32 reference of the same op.

Tolerance: the kernel feeds bf16 probabilities to the tensor cores, so the
max error is bounded at 2e-2 of the output scale. Each case runs on the
tcgen05 kernels as chosen by shape, and on the streaming tcgen05 kernel where
it applies (af_set_attention_kernel).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(q, k, v, n_heads, n_kv):
    """fp32 softmax(q k^T / sqrt(128)) v per head; q [n, nh*128], k/v [n, T, nkv*128]."""
    n = q.shape[0]
    grp = n_heads // n_kv
    qh = q.float().view(n, n_heads, 128)
    kh = k.float().view(n, -1, n_kv, 128).repeat_interleave(grp, dim=2)
    vh = v.float().view(n, -1, n_kv, 128).repeat_interleave(grp, dim=2)
    s = torch.einsum("nhd,nthd->nht", qh, kh) / 128 ** 0.5
    p = torch.softmax(s, dim=-1)
    return torch.einsum("nht,nthd->nhd", p, vh).reshape(n, -1)


def _err(a, b):
    return float((a.float() - b.float()).abs().max() / b.float().abs().max())


@pytest.fixture(params=["tc", "stream"])
def impl(request):
    """tcgen05 kernels with the shape-based choice, and the streaming kernel
    forced wherever it applies (contiguous queries, no candidate keys)."""
    from actfold_b200 import _lib

    lib = _lib.load()
    _lib.check(lib.af_set_attention_kernel(1 if request.param == "stream" else 0))
    yield request.param
    _lib.check(lib.af_set_attention_kernel(0))


@pytest.mark.parametrize("T,n_q,heads,kv", [(64, 64, 2, 2), (1024, 1024, 4, 4), (200, 37, 4, 1), (512, 130, 8, 2),
                                            (3000, 200, 2, 2), (130, 129, 32, 32)])
def test_dense_attention(T, n_q, heads, kv, impl):
    from actfold_b200.kernels import attention

    g = torch.Generator(device="cuda").manual_seed(T + n_q)
    q = torch.randn(n_q, heads * 128, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(T, kv * 128, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(T, kv * 128, device="cuda", generator=g).to(torch.bfloat16)
    out = attention(q, k, v, heads, kv)
    ref = _ref(q, k[None].expand(n_q, -1, -1), v[None].expand(n_q, -1, -1), heads, kv)
    assert _err(out, ref) <= 2e-2


def _fresh_case(T, heads, kv, fresh, qsel, seed=0):
    """Parent K/V plus per-child fresh K/V rows; queries are candidate rows qsel.

    Returns the kernel inputs and the fp32 reference output of every query.
    """
    g = torch.Generator(device="cuda").manual_seed(seed)
    D = kv * 128
    pk = torch.randn(T, D, device="cuda", generator=g).to(torch.bfloat16)
    pv = torch.randn(T, D, device="cuda", generator=g).to(torch.bfloat16)
    C = max(fresh) + 1
    cand = [(c, t) for c in range(C) for t in fresh.get(c, [])]
    nc = len(cand)
    fk = torch.randn(nc, D, device="cuda", generator=g).to(torch.bfloat16)
    fv = torch.randn(nc, D, device="cuda", generator=g).to(torch.bfloat16)
    fchild = torch.tensor([c for c, _ in cand], dtype=torch.int32, device="cuda")
    bits_np = np.zeros((C, (T + 31) // 32), np.uint32)
    for c, t in cand:
        bits_np[c, t // 32] |= np.uint32(1 << (t % 32))
    bits = torch.from_numpy(bits_np.view(np.int32)).cuda()
    qall = torch.randn(nc, heads * 128, device="cuda", generator=g).to(torch.bfloat16)
    qsrc = torch.tensor(qsel, dtype=torch.int32, device="cuda")
    qchild = torch.tensor([cand[i][0] for i in qsel], dtype=torch.int32, device="cuda")
    # reference: per query, parent K/V with the child's fresh rows replaced
    ks, vs = [], []
    for i in qsel:
        c = cand[i][0]
        k = pk.clone()
        v = pv.clone()
        for j, (cc, t) in enumerate(cand):
            if cc == c:
                k[t] = fk[j]
                v[t] = fv[j]
        ks.append(k)
        vs.append(v)
    ref = _ref(qall[qsrc.long()], torch.stack(ks), torch.stack(vs), heads, kv)
    args = dict(qsrc=qsrc, qchild=qchild, fresh_bits=bits, fk=fk, fv=fv, fchild=fchild)
    return qall, pk, pv, args, ref


@pytest.mark.parametrize("kv", [4, 2])
def test_fresh_key_overrides(kv, impl):
    from actfold_b200.kernels import attention

    heads = 4
    fresh = {0: [3, 77, 299], 1: [0, 150], 2: [5, 6, 7, 8, 200]}
    qsel = [0, 2, 3, 5, 6, 9]
    qall, pk, pv, args, ref = _fresh_case(300, heads, kv, fresh, qsel)
    out = attention(qall, pk, pv, heads, kv, **args)
    assert _err(out, ref) <= 2e-2
    # dynamic counts: only the first 4 queries are valid
    out2 = torch.zeros_like(out)
    n_q = torch.tensor([4], dtype=torch.int32, device="cuda")
    attention(qall, pk, pv, heads, kv, out=out2, n_q=n_q, **args)
    assert _err(out2[:4], ref[:4]) <= 2e-2
    assert (out2[4:] == 0).all()


@pytest.mark.parametrize("T", [300, 1024])
def test_key_splits_over_a_cluster(T, impl):
    """Key splits combined over a cluster give the reference result: 70 queries
    leave the query tile partly empty, and a dynamic query count cuts it further."""
    from actfold_b200.kernels import attention

    heads, kv = 4, 2
    fresh = {0: [1, 64, T - 1], 1: [0, 127, 128], 2: list(range(10, 30)), 3: [T // 2]}
    nc = sum(len(v) for v in fresh.values())
    qsel = [i % nc for i in range(70)]
    qall, pk, pv, args, ref = _fresh_case(T, heads, kv, fresh, qsel, seed=T)
    out = attention(qall, pk, pv, heads, kv, **args)
    assert _err(out, ref) <= 2e-2
    out2 = torch.zeros_like(out)
    n_q = torch.tensor([67], dtype=torch.int32, device="cuda")
    attention(qall, pk, pv, heads, kv, out=out2, n_q=n_q, **args)
    assert _err(out2[:67], ref[:67]) <= 2e-2
    assert (out2[67:] == 0).all()


def test_fold_shape_many_children_and_timeout_status(impl):
    """The folded pass's shape (128 packed queries, 1024 parent keys, 128 candidate keys of 8
    children, 32 heads) against the reference, with a status word that stays clear."""
    from actfold_b200.kernels import DeviceStatus, attention

    heads, kv, T = 32, 32, 1024
    g = torch.Generator().manual_seed(5)
    fresh = {c: sorted(torch.randperm(T, generator=g)[:16].tolist()) for c in range(8)}
    qsel = list(range(128))
    qall, pk, pv, args, ref = _fresh_case(T, heads, kv, fresh, qsel, seed=11)
    st = DeviceStatus()
    out = attention(qall, pk, pv, heads, kv, status=st, **args)
    torch.cuda.synchronize()
    st.check_status()
    assert _err(out, ref) <= 2e-2


def test_unsupported_shape_is_refused_before_launch():
    """Gathered queries over more than 24 key blocks fit neither tcgen05 kernel: the call raises ValueError (AF_ERR_ARG,
    checked on the host before any launch) instead of running anything."""
    from actfold_b200.kernels import attention

    T, heads = 25 * 128, 2
    q = torch.zeros(4, heads * 128, device="cuda", dtype=torch.bfloat16)
    k = torch.zeros(T, heads * 128, device="cuda", dtype=torch.bfloat16)
    qsrc = torch.tensor([3, 2, 1, 0], dtype=torch.int32, device="cuda")
    with pytest.raises(ValueError, match="24 key blocks"):
        attention(q, k, k, heads, heads, qsrc=qsrc)
    torch.cuda.synchronize()
