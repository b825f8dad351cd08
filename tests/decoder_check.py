"""Token- and logit-level parity checks shared by the decoder tests.

The CPU reference (oracle/llama_ref.py, TR's GPT step over the oracle's
float-path product) is fed the GPU's own token history, one token per step,
so every generated position is checked against the reference's logits for
exactly the context the GPU saw:

  * logits: relative L2 <= TOL at every step that has GPU logits;
  * tokens: at every generated position the GPU's token is the reference's
    first maximum, or its reference logit is within TOL * max|logit| of that
    maximum (a tie at float precision, counted and returned).

tol replaces TOL for paths whose operands are rounded to fp16 on purpose
(the prompt pass's tensor-core products and attention).

Nothing is skipped after a mismatch: a token outside the tie band fails the
check at the position where it happens.
"""
from __future__ import annotations

import numpy as np

TOL = 1e-3


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def distinct_generated(tokens, n_prompt: int) -> int:
    return len(set(int(t) for t in tokens[n_prompt:]))


def check_history(host: dict, tokens, n_prompt: int, gpu_logits: dict | None = None, tol: float = TOL) -> dict:
    """Feed tokens[0..n-2] to a fresh reference decoder and check the GPU
    history `tokens` (prompt, then greedy) position by position.

    gpu_logits maps a step position p (the step that fed tokens[p]) to the
    GPU's logits of that step.  Returns {"ties": [...], "max_rel_l2": x,
    "checked_tokens": k, "checked_logits": j}."""
    from oracle.llama_ref import Reference

    ref = Reference(host)
    tokens = [int(t) for t in tokens]
    ties, worst, nt, nl = [], 0.0, 0, 0
    for pos in range(len(tokens) - 1):
        lg = ref.step(tokens[pos], pos)
        if gpu_logits is not None and pos in gpu_logits:
            e = rel_l2(gpu_logits[pos], lg)
            assert e <= tol, f"logits at position {pos}: rel-L2 {e:.3e}"
            worst = max(worst, e)
            nl += 1
        nxt = pos + 1
        if nxt < n_prompt:
            continue
        best = int(np.argmax(lg))
        got = tokens[nxt]
        nt += 1
        if got != best:
            band = tol * float(np.abs(lg).max())
            gap = float(lg[best] - lg[got])
            assert gap < band, f"token at position {nxt}: {got} (reference {best}, gap {gap:.4g} > tie band {band:.4g})"
            ties.append(nxt)
    return {"ties": ties, "max_rel_l2": worst, "checked_tokens": nt, "checked_logits": nl}


def min_margin_ratio(logits, margins, n_prompt: int) -> float:
    """Smallest top-2 margin of the reference's own greedy picks, relative to
    that step's max|logit| (inf margins mark prompt steps)."""
    r = [m / float(np.abs(lg).max()) for lg, m in zip(logits, margins) if np.isfinite(m)]
    return min(r) if r else float("inf")
