"""Block decoding with folded verification steps, restated in numpy (TEST INFRASTRUCTURE).

The reference has no folded block-decoding loop (its Fast-dLLM sampler,
actfold/models/fast_dllm_sampler.py:111-242, verifies nothing and passes
parent_branch_id=None), so this oracle is defined step by step from the
reference's own pieces:

  * each step's children are folded against the current parent exactly as
    FoldedModel does for a child (``oracle.folding.llada_folded_children``);
  * the accepted child becomes the next parent with its merged per-layer
    states, as the reference's cache stores a verified child
    (``oracle.folding.llada_promote``);
  * the draft, the child construction (child i unmasks the edits[i] most
    confident masked positions of the block) and the acceptance rule (most
    unmasked positions among the children whose mean stable ratio reaches the
    acceptance threshold and that unmask no more positions than the
    confidence-threshold rule of fast_dllm_sampler.py:185-189 allows, at least
    min(min_edits, largest child)) are restated here with plain loops.
"""

from __future__ import annotations

import numpy as np

from oracle import folding as OF


def block_decode(prompt, weights, dims, cfg, draft, mask_id: int, max_steps: int | None = None) -> dict:
    """Returns the final canvas, the accepted child and unmasked count per step, and the final parent."""
    canvas = np.concatenate([np.asarray(prompt, np.int64), np.full(cfg.gen_len, mask_id, np.int64)])
    parent = OF.llada_parent(canvas, weights, dims)
    C = cfg.n_children
    if C == 1:
        edits = [cfg.min_edits]
    else:
        edits = [int(np.rint(cfg.min_edits + (cfg.max_edits - cfg.min_edits) * i / (C - 1))) for i in range(C)]
    step = 0
    accepted, unmasked = [], []
    for b in range(cfg.gen_len // cfg.block_size):
        lo = cfg.prompt_len + b * cfg.block_size
        while max_steps is None or step < max_steps:
            masked = [p for p in range(lo, lo + cfg.block_size) if canvas[p] == mask_id]
            if not masked:
                break
            tokens, conf = draft(step, np.array(masked))
            ranked = sorted(range(len(masked)), key=lambda j: (-conf[j], j))
            children, n = [], []
            for e in edits:
                k = min(e, len(masked))
                child = canvas.copy()
                for j in ranked[:k]:
                    child[masked[j]] = tokens[j]
                children.append(child)
                n.append(k)
            children = np.stack(children)
            res = OF.llada_folded_children(children, parent, weights, dims, cfg.tau)
            ratio = res["masks"].mean(axis=(0, 2))  # [C]: mean over layers and tokens
            allowed = max(sum(1 for c in conf if c > cfg.threshold), 1, min(cfg.min_edits, max(n)))
            ok = [i for i in range(C) if n[i] <= allowed and ratio[i] >= cfg.acceptance_threshold]
            if not ok:
                ok = [i for i in range(C) if n[i] <= allowed]
            best = max(n[i] for i in ok)
            i = min(i for i in ok if n[i] == best)
            parent = OF.llada_promote(res, i)
            canvas = children[i].copy()
            accepted.append(i)
            unmasked.append(n[i])
            step += 1
        if max_steps is not None and step >= max_steps:
            break
    return {"tokens": canvas, "accepted": accepted, "unmasked": unmasked, "parent": parent, "steps": step}
