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


def fp16_prompt_deviation(host: dict, prompt) -> float:
    """How far the reference's logits after `prompt` move when the operands
    the prompt pass rounds to fp16 are rounded: every layer product's
    activations and dequantised weights (qkv, o, gate_up, down), the
    attention's scaled q and its softmax weights P.  Relative L2 of the last
    step's logits, rounded against exact."""
    import oracle.llama_ref as LR
    from oracle import oracle as O

    class Rounded(LR.Reference):
        def __init__(self, model):
            super().__init__(model)
            D = model["cfg"].d_model
            c = model["cfg"]
            K = {"qkv": D, "o": c.n_heads * c.head_dim, "gate_up": D, "down": c.ffn_dim}
            self.w16 = {k: [O.dequant(LR.TYPES[k], w).reshape(-1, K[k]).astype(np.float16).astype(np.float64)
                            for w in model[k]] for k in K}

        def mv(self, kind, l, x):
            return (self.w16[kind][l] @ x.astype(np.float16).astype(np.float64)).astype(np.float32)

        def step(self, token, pos):
            c, m = self.c, self.m
            H, KVH, hd, D, F = c.n_heads, c.n_kv_heads, c.head_dim, c.d_model, c.ffn_dim
            half, G = hd // 2, c.n_heads // c.n_kv_heads
            x = O.embedding(LR.TYPES["tok_emb"], m["tok_emb"], D, [token])[0].astype(np.float32)
            for l in range(c.n_layers):
                h = LR.rms(x, m["attn_norm"][l], c.eps)
                qkv = self.mv("qkv", l, h).reshape(H + 2 * KVH, hd)
                a, b = qkv[:H + KVH, :half], qkv[:H + KVH, half:]
                cs, sn = self.cos[pos], self.sin[pos]
                rot = np.concatenate([a * cs - b * sn, a * sn + b * cs], axis=1).astype(np.float32)
                q = rot[:H]
                self.kc[l, :, pos] = rot[H:H + KVH].astype(np.float16)
                self.vc[l, :, pos] = qkv[H + KVH:].astype(np.float16)
                att = np.empty((H, hd), np.float32)
                sc = np.float32(np.log2(np.e) / np.sqrt(np.float32(hd)))
                for hh in range(H):
                    k = self.kc[l, hh // G, :pos + 1].astype(np.float32)
                    v = self.vc[l, hh // G, :pos + 1].astype(np.float32)
                    s_ = k @ (q[hh] * sc).astype(np.float16).astype(np.float32)
                    p = np.exp2(s_ - s_.max()).astype(np.float16).astype(np.float32)
                    att[hh] = (p @ v) / p.sum()
                x = (x + self.mv("o", l, att.reshape(-1))).astype(np.float32)
                h = LR.rms(x, m["ffn_norm"][l], c.eps)
                gu = self.mv("gate_up", l, h)
                g, u = gu[:F], gu[F:]
                with np.errstate(over="ignore"):
                    act = (g / (np.float32(1.0) + np.exp(-g)) * u).astype(np.float32)
                x = (x + self.mv("down", l, act)).astype(np.float32)
            return LR.matvec("head", m["head"], LR.rms(x, m["final_norm"], c.eps), c.vocab)

    def last(ref):
        lg = None
        for pos, t in enumerate(prompt):
            lg = ref.step(int(t), pos)
        return lg

    return rel_l2(last(Rounded(host)), last(LR.Reference(host)))
