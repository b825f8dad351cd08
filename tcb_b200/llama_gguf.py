"""Llama-shaped decoders as GGUF files: write a model (random-init ones
included) with llama.cpp's tensor names and read it back for the engine.

The mapping follows TR's GGUF model loader (lib/pretrained.tr 95-130,
_gguf_blok 276-316; internal/stdlib/ml/load_gguf.go 20-120):

  token_embd.weight            [vocab, d]      -> tok_emb
  blk.N.attn_norm.weight       [d]  F32        -> attn_norm[N]
  blk.N.attn_q / attn_k / attn_v.weight        -> qkv[N] (rows q, then k, then v)
  blk.N.attn_output.weight     [d, H hd]       -> o[N]
  blk.N.ffn_norm.weight        [d]  F32        -> ffn_norm[N]
  blk.N.ffn_gate / ffn_up.weight               -> gate_up[N] (rows gate, then up)
  blk.N.ffn_down.weight        [d, ffn]        -> down[N]
  output_norm.weight           [d]  F32        -> final_norm
  output.weight                [vocab, d]      -> head

GGUF dims are the reverse of the shape (dims[0] is the innermost axis).  The
converter stores the rows of attn_q and attn_k of every head interleaved
(llama.cpp rotates adjacent pairs, TR and this engine rotate halves): file row
h*hd + 2r holds row r of the head and h*hd + 2r + 1 holds row r + hd/2.  The
writer applies that order and the loader undoes it (TR's _gguf_satır_sırası).
Quantized tensors are kept as their verbatim blocks; every one is checked for
NaN/Inf fp16 scales on load (TR's CheckQuantScales).  Block types are taken
per tensor, as TR's loader does (pretrained.tr 85-141): any of Q8_0, Q4_0,
Q4_K, Q6_K for the embedding, the head and each layer's products, with
attn_q/attn_k of one type and ffn_gate/ffn_up of one type (they are merged
into one product each); attn_v and ffn_down may differ per layer, as in
llama.cpp's Q4_K_M files.  Types other than the engine's defaults
(llama.TYPES) are recorded in the model's "types".  Norms are F32.
"""
from __future__ import annotations

import mmap

import numpy as np

from . import BLOCK, TcbError, check_scales
from . import gguf as G
from .llama import LAYER_KINDS, TYPES, LlamaConfig, layer_types, qkv_split

ARCH = "llama"


def _qk_file_order(heads: int, hd: int) -> np.ndarray:
    """For engine row j (head h, row r), the file row holding it."""
    r = np.arange(hd)
    within = np.where(r < hd // 2, 2 * r, 2 * (r - hd // 2) + 1)
    return (np.arange(heads)[:, None] * hd + within[None, :]).reshape(-1)


def _rows(a: np.ndarray, n_rows: int) -> np.ndarray:
    return np.asarray(a, dtype=np.uint8).reshape(n_rows, -1)


def write(path: str, cfg: LlamaConfig, host: dict, context_length: int | None = None):
    """Write the host model (llama.host_model layout) as a GGUF v3 file."""
    H, KVH, hd, D, F, V = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.d_model, cfg.ffn_dim, cfg.vocab
    b = G.Builder()
    b.kv("general.architecture", ARCH).kv("general.name", "tcb random-init llama")
    for k, v in (("block_count", cfg.n_layers), ("context_length", context_length or cfg.max_ctx),
                 ("embedding_length", D), ("feed_forward_length", F), ("attention.head_count", H),
                 ("attention.head_count_kv", KVH), ("attention.key_length", hd), ("rope.dimension_count", hd),
                 ("vocab_size", V)):
        b.kv(f"{ARCH}.{k}", (G.U32, v))
    b.kv(f"{ARCH}.rope.freq_base", (G.F32V, cfg.rope_theta))
    b.kv(f"{ARCH}.attention.layer_norm_rms_epsilon", (G.F32V, cfg.eps))

    def q(name, wt, rows, K, data):
        b.tensor(name, wt, [K, rows], np.ascontiguousarray(data, dtype=np.uint8).tobytes())

    def f32(name, a):
        b.tensor(name, G.F32, [D], np.ascontiguousarray(a, dtype=np.float32).tobytes())

    types = host.get("types") or {}
    q("token_embd.weight", types.get("tok_emb", TYPES["tok_emb"]), V, D, host["tok_emb"])
    for l, (qk_t, v_t, o_t, gu_t, dn_t) in enumerate(layer_types(host)):
        p = f"blk.{l}."
        f32(p + "attn_norm.weight", host["attn_norm"][l])
        raw = np.asarray(host["qkv"][l], dtype=np.uint8)
        nqk = qkv_split(cfg, qk_t)
        qk = _rows(raw[:nqk], (H + KVH) * hd)
        qr, kr, vr = qk[:H * hd], qk[H * hd:], _rows(raw[nqk:], KVH * hd)
        fq = np.empty_like(qr)
        fq[_qk_file_order(H, hd)] = qr
        fk = np.empty_like(kr)
        fk[_qk_file_order(KVH, hd)] = kr
        q(p + "attn_q.weight", qk_t, H * hd, D, fq)
        q(p + "attn_k.weight", qk_t, KVH * hd, D, fk)
        q(p + "attn_v.weight", v_t, KVH * hd, D, vr)
        q(p + "attn_output.weight", o_t, D, H * hd, host["o"][l])
        f32(p + "ffn_norm.weight", host["ffn_norm"][l])
        gu = _rows(host["gate_up"][l], 2 * F)
        q(p + "ffn_gate.weight", gu_t, F, D, gu[:F])
        q(p + "ffn_up.weight", gu_t, F, D, gu[F:])
        q(p + "ffn_down.weight", dn_t, D, F, host["down"][l])
    f32("output_norm.weight", host["final_norm"])
    q("output.weight", types.get("head", TYPES["head"]), V, D, host["head"])
    b.write(path)


def _u(f: G.File, key: str, default=None) -> int:
    v = f.values.get(f"{ARCH}.{key}")
    if v is None:
        if default is None:
            raise ValueError(f"gguf: missing {ARCH}.{key}")
        return default
    if v.type not in (G.U8, G.U16, G.U32, G.U64, G.I8, G.I16, G.I32, G.I64) or v.data < 0:
        raise ValueError(f"gguf: {ARCH}.{key} is not a count")
    return int(v.data)


def _f(f: G.File, key: str, default=None) -> float:
    v = f.values.get(f"{ARCH}.{key}")
    if v is None:
        if default is None:
            raise ValueError(f"gguf: missing {ARCH}.{key}")
        return default
    if v.type not in (G.F32V, G.F64V):
        raise ValueError(f"gguf: {ARCH}.{key} is not a float")
    return float(v.data)


def load(path: str, max_ctx: int | None = None) -> tuple:
    """(LlamaConfig, host model) from a GGUF file written with this mapping.
    max_ctx sizes the engine's K/V cache (default: the file's context length,
    at most 4096)."""
    with open(path, "rb") as fh:
        mm = mmap.mmap(fh.fileno(), 0, access=mmap.ACCESS_READ)
    try:
        f = G.decode(mm)
        arch = f.values.get("general.architecture")
        if arch is None or arch.data != ARCH:
            raise ValueError(f"gguf: general.architecture {getattr(arch, 'data', None)!r}, not {ARCH!r}")
        split = f.values.get("split.count")
        if split is not None and int(split.data) > 1:
            raise ValueError("gguf: split files are not read")
        H, KVH = _u(f, "attention.head_count"), _u(f, "attention.head_count_kv")
        D, F, L = _u(f, "embedding_length"), _u(f, "feed_forward_length"), _u(f, "block_count")
        hd = _u(f, "attention.key_length", D // H)
        if _u(f, "rope.dimension_count", hd) != hd:
            raise ValueError("gguf: rotary over part of the head is not provided")
        V = _u(f, "vocab_size", int(f.tensor("token_embd.weight").dims[1]))
        ctx_len = _u(f, "context_length", 2048)
        cfg = LlamaConfig(n_layers=L, d_model=D, n_heads=H, n_kv_heads=KVH, head_dim=hd, ffn_dim=F, vocab=V,
                          max_ctx=max_ctx or min(ctx_len, 4096),
                          eps=_f(f, "attention.layer_norm_rms_epsilon"), rope_theta=_f(f, "rope.freq_base", 10000.0))

        qtypes = set(BLOCK)

        def get(name, quant, rows, K):
            """(bytes, type) of a quantized tensor, or the F32 vector"""
            try:
                t = f.tensor(name)
            except KeyError:
                raise ValueError(f"gguf: missing tensor {name}") from None
            if (t.type in qtypes) != quant:
                raise ValueError(f"gguf: {name} is {G.TYPES[t.type][0]}, the engine takes "
                                 f"{'Q8_0, Q4_0, Q4_K or Q6_K' if quant else 'F32'}")
            if list(t.dims) != ([K, rows] if quant else [K]):
                raise ValueError(f"gguf: {name} has dims {t.dims}")
            raw = np.frombuffer(G.tensor_bytes(mm, f, t), dtype=np.uint8).copy()
            if not quant:
                return raw.view(np.float32)
            bad = check_scales(t.type, raw)
            if bad >= 0:
                raise TcbError(10, f"gguf: {name}: block {bad} has a NaN/Inf scale")
            return raw, t.type

        emb, emb_t = get("token_embd.weight", True, V, D)
        head, head_t = get("output.weight", True, V, D)
        m = {"cfg": cfg, "tok_emb": emb, "final_norm": get("output_norm.weight", False, None, D), "head": head}
        for k in ("attn_norm", "ffn_norm", "qkv", "o", "gate_up", "down"):
            m[k] = []
        lt = {k: [] for k in LAYER_KINDS}
        inv_q, inv_k = _qk_file_order(H, hd), _qk_file_order(KVH, hd)
        for l in range(L):
            p = f"blk.{l}."
            m["attn_norm"].append(get(p + "attn_norm.weight", False, None, D))
            qb, qt = get(p + "attn_q.weight", True, H * hd, D)
            kb, kt = get(p + "attn_k.weight", True, KVH * hd, D)
            vb, vt = get(p + "attn_v.weight", True, KVH * hd, D)
            if qt != kt:
                raise ValueError(f"gguf: {p}attn_q and attn_k differ in type (merged into one product)")
            qr, kr = _rows(qb, H * hd)[inv_q], _rows(kb, KVH * hd)[inv_k]
            m["qkv"].append(np.concatenate([qr.reshape(-1), kr.reshape(-1), vb]))
            ob, ot = get(p + "attn_output.weight", True, D, H * hd)
            m["o"].append(ob)
            m["ffn_norm"].append(get(p + "ffn_norm.weight", False, None, D))
            gb, gt = get(p + "ffn_gate.weight", True, F, D)
            ub, ut = get(p + "ffn_up.weight", True, F, D)
            if gt != ut:
                raise ValueError(f"gguf: {p}ffn_gate and ffn_up differ in type (merged into one product)")
            m["gate_up"].append(np.concatenate([gb, ub]))
            db, dt = get(p + "ffn_down.weight", True, D, F)
            m["down"].append(db)
            for k, t in zip(LAYER_KINDS, (qt, vt, ot, gt, dt)):
                lt[k].append(t)
        default = dict(zip(LAYER_KINDS, layer_types({"cfg": cfg})[0])) if L else {}
        types = {k: v for k, v in lt.items() if any(t != default[k] for t in v)}
        if emb_t != TYPES["tok_emb"]:
            types["tok_emb"] = emb_t
        if head_t != TYPES["head"]:
            types["head"] = head_t
        if types:
            m["types"] = types
        return cfg, m
    finally:
        mm.close()
