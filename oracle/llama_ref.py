"""CPU reference of the Llama-shaped batch-1 decode step.

TEST INFRASTRUCTURE ONLY: the decoder parity tests use it as the checker;
the shipped library never imports it.

Restates TR's GPT step over quantized weights (sekerahmet/TCB lib/layers.tr):
  x = embed(token)                                    Embedding, 50-66
  per block: h = x + attn(rms(x)); x = h + ffn(rms(h)) TransformerBlock, 348-389
  logits = head(rms(x)); greedy = first maximum        GPT.single_step, 658-666
with
  rms(x) = x / sqrt(mean(x^2) + eps) * w               RMSNorm, 68-79
  rotary: f_i = theta^(-2i/hd) (double, then float32), angle = t * f_i in
  float32, halves (a, b) -> (a cos - b sin, a sin + b cos)   85-107
  attention: softmax(q.k / sqrt(hd)) v over positions <= t, query head h
  using KV head h // (H / KVH)                          CausalAttention, 126-215
  ffn: down(silu(g) * u) over the merged [G | U] rows   SwiGLU, 224-276
The quantized products are the oracle's restatement of TR's float path
(quantGemv: dotF32 order, tensor/cpu_quant.go:151-160) and the embedding row
is TR's exact dequant.  The K/V cache holds float16 values, as the
benchmark's decoder configuration specifies.  Everything else is float32.
"""
from __future__ import annotations

import numpy as np

from . import oracle as O

Q4_K, Q6_K = O.Q4_K, O.Q6_K
TYPES = {"tok_emb": Q4_K, "qkv": Q4_K, "o": Q6_K, "gate_up": Q4_K, "down": Q6_K, "head": Q6_K}


def rotary_tables(max_ctx: int, hd: int, theta: float):
    half = hd // 2
    f = np.array([np.float32(theta ** (-2.0 * i / hd)) for i in range(half)], np.float32)
    ang = (np.arange(max_ctx, dtype=np.float32)[:, None] * f[None, :]).astype(np.float32)
    return np.cos(ang.astype(np.float64)).astype(np.float32), np.sin(ang.astype(np.float64)).astype(np.float32)


def rms(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    ms = np.float32(np.dot(x.astype(np.float64), x.astype(np.float64)) / x.size)
    return ((x / np.sqrt(np.float32(ms + np.float32(eps)))) * w).astype(np.float32)


def matvec(kind: str, w: np.ndarray, x: np.ndarray, N: int, wt: int | None = None) -> np.ndarray:
    return O.qgemm_float(TYPES[kind] if wt is None else wt, x.reshape(1, -1).astype(np.float32), w, N)[0]


BLOCK = {O.Q8_0: (32, 34), O.Q4_0: (32, 18), Q4_K: (256, 144), Q6_K: (256, 210)}


def layer_types(model: dict, l: int) -> tuple:
    """(qk, v, o, gate_up, down) block types of layer l: model["types"] lists
    per layer (absent: the class types)."""
    t = model.get("types") or {}
    cls = {"qk": "qkv", "v": "qkv", "o": "o", "gate_up": "gate_up", "down": "down"}
    return tuple(t[k][l] if k in t else TYPES[cls[k]] for k in ("qk", "v", "o", "gate_up", "down"))


class Reference:
    """Greedy decoding with prompt feeding, one token per step."""

    def __init__(self, model: dict):
        self.m = model
        c = model["cfg"]
        self.c = c
        self.cos, self.sin = rotary_tables(c.max_ctx, c.head_dim, c.rope_theta)
        self.kc = np.zeros((c.n_layers, c.n_kv_heads, c.max_ctx, c.head_dim), np.float16)
        self.vc = np.zeros_like(self.kc)

    def step(self, token: int, pos: int):
        """logits of one step at position pos (appends K/V)."""
        c, m = self.c, self.m
        H, KVH, hd, D, F = c.n_heads, c.n_kv_heads, c.head_dim, c.d_model, c.ffn_dim
        half, G = hd // 2, c.n_heads // c.n_kv_heads
        ct = m.get("types") or {}
        x = O.embedding(ct.get("tok_emb", TYPES["tok_emb"]), m["tok_emb"], D, [token])[0].astype(np.float32)
        for l in range(c.n_layers):
            qk_t, v_t, o_t, gu_t, dn_t = layer_types(m, l)
            h = rms(x, m["attn_norm"][l], c.eps)
            if qk_t == v_t:
                qkv = matvec("qkv", m["qkv"][l], h, (H + 2 * KVH) * hd, qk_t)
            else:
                e, b = BLOCK[qk_t]
                nb = (H + KVH) * hd * (D // e) * b
                qkv = np.concatenate([matvec("qkv", m["qkv"][l][:nb], h, (H + KVH) * hd, qk_t),
                                      matvec("qkv", m["qkv"][l][nb:], h, KVH * hd, v_t)])
            qkv = qkv.reshape(H + 2 * KVH, hd)
            a, b = qkv[:H + KVH, :half], qkv[:H + KVH, half:]
            cs, sn = self.cos[pos], self.sin[pos]
            rot = np.concatenate([a * cs - b * sn, a * sn + b * cs], axis=1).astype(np.float32)
            q = rot[:H]
            self.kc[l, :, pos] = rot[H:H + KVH].astype(np.float16)
            self.vc[l, :, pos] = qkv[H + KVH:].astype(np.float16)
            att = np.empty((H, hd), np.float32)
            scale = np.float32(1.0 / np.sqrt(np.float32(hd)))
            for hh in range(H):
                kh = hh // G
                k = self.kc[l, kh, :pos + 1].astype(np.float32)
                v = self.vc[l, kh, :pos + 1].astype(np.float32)
                s = (k @ q[hh]) * scale
                p = np.exp(s - s.max())
                att[hh] = (p @ v) / p.sum()
            x = (x + matvec("o", m["o"][l], att.reshape(-1), D, o_t)).astype(np.float32)
            h = rms(x, m["ffn_norm"][l], c.eps)
            gu = matvec("gate_up", m["gate_up"][l], h, 2 * F, gu_t)
            g, u = gu[:F], gu[F:]
            with np.errstate(over="ignore"):  # exp(-g) = inf gives silu = -0, as on the device
                act = (g / (np.float32(1.0) + np.exp(-g)) * u).astype(np.float32)
            x = (x + matvec("down", m["down"][l], act, D, dn_t)).astype(np.float32)
        return matvec("head", m["head"], rms(x, m["final_norm"], c.eps), c.vocab, ct.get("head"))

    def generate(self, prompt, steps: int):
        """Token history (prompt, then greedy), the logits of every step and
        the top-2 margin of every greedy choice."""
        toks = [int(prompt[0])]
        logits, margins = [], []
        for pos in range(steps):
            lg = self.step(toks[-1], pos)
            logits.append(lg)
            if pos + 1 < len(prompt):
                toks.append(int(prompt[pos + 1]))
                margins.append(np.inf)
            else:
                top = np.argsort(lg)[::-1][:2]
                toks.append(int(np.argmax(lg)))
                margins.append(float(lg[top[0]] - lg[top[1]]))
        return np.array(toks, np.int64), logits, margins
