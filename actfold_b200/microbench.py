"""Bandwidth of the row kernels behind the drop-in API (one B200).

    python -m actfold_b200.microbench [--children 32] [--seq 1024] [--hidden 4096] [--reps 20] [--only KERNEL]

Times, through the public API, the three HBM-bound kernels that replace the
reference's per-token tensor work:

* ``gate``   SimilarityGate.forward_compact (similarity_gate.py:43-103): mask,
             divergent index lists and counts for C children against one
             parent (broadcast); algorithmic bytes = children + parent rows
             read, mask + index lists + counts written.
* ``merge``  merge_stable_divergent (fused_ops.py:206-253) with half the rows
             stable: each output row reads only its selected source row;
             bytes = C*T rows read + C*T rows written.
* ``gather`` gather_cached_activations' masked reconstruction
             (fused_ops.py:256-324) with half the rows selected: selected rows
             read, every row written (zeros elsewhere).

Beside ``merge``, the same merge done the reference's ways, on the same
tensors and with the same byte count: ``merge_torch_where`` (its torch
fallback, fused_ops.py:38-51) and ``merge_reference_triton`` (its own
``merge_stable_divergent``, which runs its Triton ``_merge_kernel`` on CUDA,
fused_ops.py:95-135, imported from the reference package installed under
``baseline/_ref`` when it is there; skipped otherwise).

Inputs are bf16 [C, T, H] (268 MB at the defaults, above the 126 MB L2). Each
kernel's calls are captured in a CUDA graph of ``reps`` launches, replayed
after warm-up and timed with CUDA events on the capturing stream; one JSON
line per kernel gives GB/s of algorithmic bytes and the fraction of the
measured copy bandwidth (MEASURED_PEAKS.json ``hbm_gbs``).
"""

from __future__ import annotations

import argparse
import json
import os

import torch

FALLBACK_HBM_GBS = 6650.0


def _peak() -> tuple[float, str]:
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def _time(fn, reps: int, rounds: int = 5) -> float:
    """Mean microseconds per call: `reps` calls captured in one graph, best of `rounds` replays."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            fn()
    g.replay()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(rounds):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1) * 1e3 / reps)
    return best


def _reference_merge():
    """The reference's merge_stable_divergent from baseline/_ref, or (None, reason)."""
    import sys
    import tempfile

    ref = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "actfold")):
        return None, "reference package not installed under baseline/_ref"
    # The reference package imports matplotlib / seaborn (for its plots) on import; neither is
    # installed here, so empty stand-ins go on the path first. Nothing of them is used.
    shim = tempfile.mkdtemp(prefix="af_ref_shim_")
    for name, body in (("matplotlib", "def use(*a, **k):\n    pass\n"), ("seaborn", "")):
        os.makedirs(os.path.join(shim, name))
        with open(os.path.join(shim, name, "__init__.py"), "w") as f:
            f.write(body)
    with open(os.path.join(shim, "matplotlib", "pyplot.py"), "w") as f:
        f.write("def __getattr__(name):\n    raise AttributeError(name)\n")
    sys.path[:0] = [shim, ref]
    # Triton 3.6 rejects the kernel's non-constexpr global annotations unless told to accept them.
    os.environ.setdefault("TRITON_ALLOW_NON_CONSTEXPR_GLOBALS", "1")
    try:
        from actfold.core.fused_ops import merge_stable_divergent as ref_merge
    except Exception as exc:  # reported in the output line, not raised
        return None, f"reference import failed: {exc}"
    return ref_merge, "baseline/_ref"


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--children", type=int, default=32)
    ap.add_argument("--seq", type=int, default=1024)
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--only", choices=["gate", "merge", "merge_torch_where", "merge_reference_triton", "gather"],
                    default=None, help="time one kernel")
    a = ap.parse_args()

    from actfold_b200.core import SimilarityGate, merge_stable_divergent
    from actfold_b200.core.fused_ops import masked_rows

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    C, T, H = a.children, a.seq, a.hidden
    g = torch.Generator(device=dev).manual_seed(0)
    child = torch.randn((C, T, H), generator=g, device=dev).to(torch.bfloat16)
    parent = torch.randn((1, T, H), generator=g, device=dev).to(torch.bfloat16)
    other = torch.randn((C, T, H), generator=g, device=dev).to(torch.bfloat16)
    half = torch.rand((C, T), generator=g, device=dev) < 0.5
    peak, src = _peak()
    row = H * 2
    gate = SimilarityGate(0.95)
    pexp = parent.expand(C, T, H)
    cases = {
        "gate": (lambda: gate.forward_compact(child, pexp), C * T * row + T * row + C * T * (1 + 4) + C * 4),
        "merge": (lambda: merge_stable_divergent(other, child, half), 2 * C * T * row),
        "merge_torch_where": (lambda: torch.where(half[..., None], other, child), 2 * C * T * row),
        "gather": (lambda: masked_rows(child, half), int(half.sum()) * row + C * T * row),
    }
    if a.only in (None, "merge_reference_triton"):
        ref_merge, why = _reference_merge()
        if ref_merge is None:
            print(json.dumps({"kernel": "merge_reference_triton", "skipped": why}), flush=True)
        else:
            cases["merge_reference_triton"] = (lambda: ref_merge(other, child, half), 2 * C * T * row)
    for name, (fn, nbytes) in cases.items():
        if a.only and name != a.only:
            continue
        try:
            us = _time(fn, a.reps)
        except Exception as exc:  # the reference's kernel on this toolchain: reported, not raised
            if name != "merge_reference_triton":
                raise
            print(json.dumps({"kernel": name, "skipped": f"{type(exc).__name__}: {str(exc).splitlines()[0][:200]}"}),
                  flush=True)
            continue
        gbs = nbytes / (us * 1e-6) / 1e9
        print(json.dumps({"kernel": name, "children": C, "seq": T, "hidden": H, "dtype": "bf16",
                          "us_per_call": round(us, 2), "algorithmic_bytes": nbytes, "achieved_gbs": round(gbs, 1),
                          "peak_gbs": peak, "peak_source": src, "frac": round(gbs / peak, 3)}), flush=True)


if __name__ == "__main__":
    main()
