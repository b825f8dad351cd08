"""Llama-shaped batch-1 decoder over quantized weights (include/tcb.h,
tcb_llama_*): a thin ctypes view plus seeded synthetic models.

Layout of a model's weights (all device tensors):
  tok_emb   [vocab, d]            Q4_K blocks
  qkv[l]    [(H + 2 KVH) hd, d]   Q4_K   (q rows, then k rows, then v rows)
  o[l]      [d, H hd]             Q6_K
  gate_up[l][2 ffn, d]            Q4_K   (gate rows, then up rows)
  down[l]   [d, ffn]              Q6_K
  head      [vocab, d]            Q6_K
  attn_norm[l], ffn_norm[l], final_norm: float32 [d]
This is the Q4_K_M assignment of the benchmark's 8B configuration (Q4_K for
attention and MLP weights, Q6_K for o_proj, down_proj and the head).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import BLOCK, Q4_0, Q4_K, Q6_K, Q8_0, TcbError, _stream, lib
from . import synth


@dataclass(frozen=True)
class LlamaConfig:
    n_layers: int
    d_model: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn_dim: int
    vocab: int
    max_ctx: int
    eps: float = 1e-5
    rope_theta: float = 500000.0


LLAMA3_8B = LlamaConfig(32, 4096, 32, 8, 128, 14336, 128256, 768)
LLAMA3_70B = LlamaConfig(80, 8192, 64, 8, 128, 28672, 128256, 1024 + 128 + 1)
TYPES = {"tok_emb": Q4_K, "qkv": Q4_K, "o": Q6_K, "gate_up": Q4_K, "down": Q6_K, "head": Q6_K}
# Standard deviation of the fp16 block scales of a random-init decoder.  The
# matvec benchmark's |N(0, 0.01)| scales give weights of standard deviation
# 2.6 (Q4_K) and 13 (Q6_K), and 32 such layers overflow float32; these give
# weights of standard deviation ~0.02 (TR's default init_std, layers.tr
# Linear), so activations stay of order one through the stack.
D_STD = {Q4_K: 7.6e-5, Q6_K: 1.5e-5, Q8_0: 2.7e-4, Q4_0: 4.3e-3}


def shapes(cfg: LlamaConfig) -> dict:
    """(rows, K) of every quantized tensor kind."""
    H, KVH, hd, D, F = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.d_model, cfg.ffn_dim
    return {"tok_emb": (cfg.vocab, D), "qkv": ((H + 2 * KVH) * hd, D), "o": (D, H * hd),
            "gate_up": (2 * F, D), "down": (D, F), "head": (cfg.vocab, D)}


def weight_bytes_per_token(cfg: LlamaConfig) -> int:
    """Quantized weight bytes a decode step streams (every layer + head + one
    embedding row)."""
    sh = shapes(cfg)
    tot = 0
    for k in ("qkv", "o", "gate_up", "down"):
        n, kk = sh[k]
        tot += cfg.n_layers * n * kk // BLOCK[TYPES[k]][0] * BLOCK[TYPES[k]][1]
    n, kk = sh["head"]
    tot += n * kk // 256 * BLOCK[Q6_K][1]
    tot += cfg.d_model // 256 * BLOCK[Q4_K][1]
    return tot


def local_shapes(cfg: LlamaConfig, tp: int) -> dict:
    """(rows, K) of every tensor kind held by one of tp ranks."""
    H, KVH, hd, D, F = cfg.n_heads // tp, cfg.n_kv_heads // tp, cfg.head_dim, cfg.d_model, cfg.ffn_dim // tp
    return {"tok_emb": (cfg.vocab, D), "qkv": ((H + 2 * KVH) * hd, D), "o": (D, H * hd),
            "gate_up": (2 * F, D), "down": (D, F), "head": (cfg.vocab // tp, D)}


# The "varied" decoder (parity tests and the benchmark models): Q4_K blocks
# centred (mins = sub-scales, dmin = 7.5 d, so a sub-block dequantises to
# d*sc*(q - 7.5)), the qkv scales 5x and the o/down scales 2x D_STD (sharper
# attention, larger sublayer outputs), and the head's block scales in a narrow
# band.  With the plain blocks a random decoder's greedy continuation
# collapses onto one or two tokens; this one visits tens of distinct tokens in
# 64 steps, so token-level parity checks the attention over a growing context.
VARIED_SCALE = {"qkv": 5.0, "o": 2.0, "down": 2.0}
VARIED_HEAD_BAND = (1.0e-5, 1.4e-5)
KINDS = ("tok_emb", "head", "qkv", "o", "gate_up", "down")


def _rows(a, kind: str, K: int, r0: int, r1: int):
    """rows [r0, r1) of a block store with K columns"""
    e, b = BLOCK[TYPES[kind]]
    rb = K // e * b
    return a[r0 * rb:r1 * rb]


def _cols(a, kind: str, N: int, K: int, k0: int, k1: int):
    """columns [k0, k1) (block aligned) of a block store of N rows"""
    e, b = BLOCK[TYPES[kind]]
    return a.reshape(N, K // e, b)[:, k0 // e:k1 // e].reshape(-1)


def _cat(parts):
    if isinstance(parts[0], np.ndarray):
        return np.concatenate(parts)
    import torch

    return torch.cat(parts).contiguous()


def shard_tensor(cfg: LlamaConfig, kind: str, w, tp: int, r: int):
    """Rank r's part of one global weight (numpy array or torch tensor) for
    tensor parallelism over tp ranks: column-parallel qkv (its query heads and
    their KV heads) and gate/up (its rows of each half), row-parallel (K-split)
    o and down, vocabulary-parallel head; the embedding and the norms are
    replicated (returned as they are)."""
    if tp == 1 or kind in ("tok_emb", "attn_norm", "ffn_norm", "final_norm"):
        return w
    H, KVH, hd, D, F, V = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.d_model, cfg.ffn_dim, cfg.vocab
    h, kv, f, v = H // tp, KVH // tp, F // tp, V // tp
    if kind == "head":
        return _rows(w, "head", D, r * v, (r + 1) * v)
    if kind == "qkv":
        return _cat([_rows(w, "qkv", D, r * h * hd, (r + 1) * h * hd),
                     _rows(w, "qkv", D, (H + r * kv) * hd, (H + (r + 1) * kv) * hd),
                     _rows(w, "qkv", D, (H + KVH + r * kv) * hd, (H + KVH + (r + 1) * kv) * hd)])
    if kind == "o":
        return _cols(w, "o", D, H * hd, r * h * hd, (r + 1) * h * hd)
    if kind == "gate_up":
        return _cat([_rows(w, "gate_up", D, r * f, (r + 1) * f), _rows(w, "gate_up", D, F + r * f, F + (r + 1) * f)])
    if kind == "down":
        return _cols(w, "down", D, F, r * f, (r + 1) * f)
    raise ValueError(kind)


def shard(cfg: LlamaConfig, model: dict, tp: int, r: int) -> dict:
    """Rank r's part of a host model for tensor parallelism over tp ranks
    (shard_tensor applied to every tensor)."""
    if tp == 1:
        return model
    out = {"cfg": cfg}
    for k, v in model.items():
        if k == "cfg":
            continue
        if k in ("tok_emb", "attn_norm", "ffn_norm", "final_norm"):
            out[k] = v  # replicated
        else:
            out[k] = [shard_tensor(cfg, k, x, tp, r) for x in v] if isinstance(v, list) else shard_tensor(cfg, k, v, tp, r)
    return out


def _d_std(kind: str, varied: bool, wt: int | None = None) -> float:
    return D_STD[TYPES[kind] if wt is None else wt] * (VARIED_SCALE.get(kind, 1.0) if varied else 1.0)


# Per-layer block types (llama.cpp's Q4_K_M files mix Q4_K and Q6_K across
# layers for the v rows and down): model["types"] maps each of these names to
# a list of n_layers types; absent names take the class type (TYPES).
LAYER_KINDS = ("qk", "v", "o", "gate_up", "down")
_CLASS_OF = {"qk": "qkv", "v": "qkv", "o": "o", "gate_up": "gate_up", "down": "down"}


def layer_types(model: dict) -> list:
    """(qk, v, o, gate_up, down) block types of every layer."""
    t = model.get("types") or {}
    L = model["cfg"].n_layers
    return [tuple(t[k][l] if k in t else TYPES[_CLASS_OF[k]] for k in LAYER_KINDS) for l in range(L)]


def qkv_split(cfg: LlamaConfig, qk_type: int) -> int:
    """Bytes of the q and k rows at the start of a layer's qkv tensor."""
    e, b = BLOCK[qk_type]
    return (cfg.n_heads + cfg.n_kv_heads) * cfg.head_dim * (cfg.d_model // e) * b


def host_model(cfg: LlamaConfig, seed: int, varied: bool = False, types: dict | None = None) -> dict:
    """Seeded model as numpy arrays (small configurations: parity tests).
    types: per-layer block types (LAYER_KINDS -> n_layers types), e.g. a
    llama.cpp Q4_K_M-like mix; a layer whose v type differs from its q/k
    type holds its v rows in that type after the q and k rows."""
    sh = shapes(cfg)
    m = {"cfg": cfg}
    rng = np.random.default_rng(seed)
    s = seed * 1000

    def w(kind, sd, wt=None, rows=None):
        wt = TYPES[kind] if wt is None else wt
        n, k = sh[kind]
        return synth.weight(wt, n if rows is None else rows, k, sd, _d_std(kind, varied, wt),
                            centered=varied and wt == Q4_K, d_band=VARIED_HEAD_BAND if varied and kind == "head" else None)

    m["tok_emb"] = w("tok_emb", s + 1)
    m["head"] = w("head", s + 2)
    m["final_norm"] = (1.0 + 0.1 * rng.standard_normal(cfg.d_model)).astype(np.float32)
    for k in ("attn_norm", "ffn_norm"):
        m[k] = [(1.0 + 0.1 * rng.standard_normal(cfg.d_model)).astype(np.float32) for _ in range(cfg.n_layers)]
    if types:
        m["types"] = {k: list(v) for k, v in types.items()}
    lt = layer_types(m)
    hd, H, KVH = cfg.head_dim, cfg.n_heads, cfg.n_kv_heads
    m["qkv"], m["o"], m["gate_up"], m["down"] = [], [], [], []
    for l in range(cfg.n_layers):
        qk_t, v_t, o_t, gu_t, dn_t = lt[l]
        sd = s + 10 + 4 * l
        if qk_t == v_t:
            m["qkv"].append(w("qkv", sd, qk_t))
        else:
            m["qkv"].append(np.concatenate([w("qkv", sd, qk_t, (H + KVH) * hd), w("qkv", sd + 500000, v_t, KVH * hd)]))
        m["o"].append(w("o", sd + 1, o_t))
        m["gate_up"].append(w("gate_up", sd + 2, gu_t))
        m["down"].append(w("down", sd + 3, dn_t))
    return m


def device_model(cfg: LlamaConfig, seed: int, host: dict | None = None, tp: tuple = (1, 0),
                 varied: bool = False) -> dict:
    """This rank's part of a model on the current CUDA device: uploads `host`
    (sharded) if given, else generates it on the GPU (fp16 block scales
    |N(0, D_STD)|, every other byte uniform; `varied` as host_model).

    Generated models are one model at every tensor-parallel degree: each
    global tensor is drawn from its own counter-based (Philox) CUDA generator
    seeded by (seed, tensor), and a rank keeps its slice of it
    (shard_tensor).  Replicated tensors are byte-identical on every rank, and
    rank r of tp holds the same bytes as the matching slice of the tp = 1
    model."""
    import torch

    def up(a):
        return torch.from_numpy(np.ascontiguousarray(a)).cuda()

    if host is not None:
        if host.get("types") and tp[0] > 1:
            raise NotImplementedError("tensor-parallel shards of a model with per-layer block types")
        host = shard(cfg, host, *tp)
        d = {"cfg": cfg}
        for k, v in host.items():
            if k == "cfg":
                continue
            if k == "types":
                d[k] = v
                continue
            d[k] = [up(x) for x in v] if isinstance(v, list) else up(v)
        return d
    sh = shapes(cfg)
    gen = torch.Generator(device="cuda")

    def seeded(tid: int):
        gen.manual_seed((seed * 1000003 + tid) & 0x7FFFFFFFFFFFFFFF)
        return gen

    def blocks(kind, tid):
        g = seeded(tid)
        wt = TYPES[kind]
        n, k = sh[kind]
        e, size = BLOCK[wt]
        nb = n * k // e
        out = torch.randint(0, 256, (nb, size), dtype=torch.uint8, device="cuda", generator=g)
        sd = _d_std(kind, varied)
        if wt == Q4_K:
            out[:, 0:4] = (torch.randn(nb, 2, device="cuda", generator=g).abs() * sd).half().view(torch.uint8)
            if varied:
                # mins = sub-scales (get_scale_min_k4 packing), dmin = 7.5 d
                out[:, 8:12] = (out[:, 8:12] & 0x0F) | ((out[:, 8:12] & 0x0F) << 4)
                out[:, 4:8] = out[:, 0:4]
                d = out[:, 0:2].contiguous().view(torch.float16).float()
                out[:, 2:4] = (d * 7.5).half().view(torch.uint8)
        elif wt == Q6_K:
            if varied and kind == "head":
                lo, hi = VARIED_HEAD_BAND
                dv = lo + (hi - lo) * torch.rand(nb, 1, device="cuda", generator=g)
            else:
                dv = torch.randn(nb, 1, device="cuda", generator=g).abs() * sd
            out[:, 208:210] = dv.half().view(torch.uint8)
        out = out.reshape(-1)
        local = shard_tensor(cfg, kind, out, *tp)
        if local.numel() != out.numel() and local.untyped_storage().data_ptr() == out.untyped_storage().data_ptr():
            local = local.clone()  # a view would keep the whole global tensor alive
        return local

    def norm(tid):
        return 1.0 + 0.1 * torch.randn(cfg.d_model, device="cuda", generator=seeded(tid))

    L = cfg.n_layers
    d = {"cfg": cfg, "tok_emb": blocks("tok_emb", 1), "head": blocks("head", 2), "final_norm": norm(3)}
    d["attn_norm"] = [norm(16 + 8 * l) for l in range(L)]
    d["ffn_norm"] = [norm(17 + 8 * l) for l in range(L)]
    for j, k in enumerate(("qkv", "o", "gate_up", "down")):
        d[k] = [blocks(k, 18 + j + 8 * l) for l in range(L)]
    return d


class _Cfg(ctypes.Structure):
    _fields_ = [("n_layers", ctypes.c_int), ("d_model", ctypes.c_int), ("n_heads", ctypes.c_int),
                ("n_kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int), ("ffn_dim", ctypes.c_int),
                ("vocab", ctypes.c_int), ("max_ctx", ctypes.c_int), ("eps", ctypes.c_float),
                ("rope_theta", ctypes.c_float), ("tp_size", ctypes.c_int), ("tp_rank", ctypes.c_int)]


_PP = ctypes.POINTER(ctypes.c_void_p)


class _Weights(ctypes.Structure):
    _fields_ = [("tok_emb", ctypes.c_void_p), ("tok_emb_type", ctypes.c_int), ("final_norm", ctypes.c_void_p),
                ("head", ctypes.c_void_p), ("head_type", ctypes.c_int), ("attn_norm", _PP), ("ffn_norm", _PP),
                ("qkv", _PP), ("qkv_type", ctypes.c_int), ("o", _PP), ("o_type", ctypes.c_int),
                ("gate_up", _PP), ("gate_up_type", ctypes.c_int), ("down", _PP), ("down_type", ctypes.c_int),
                ("layer_types", ctypes.POINTER(ctypes.c_int))]


def _bind():
    L = lib()
    if getattr(L, "_llama_bound", False):
        return L
    P = ctypes.c_void_p
    L.tcb_llama_create.argtypes = [P, ctypes.POINTER(_Cfg), ctypes.POINTER(_Weights), ctypes.POINTER(P)]
    L.tcb_llama_destroy.argtypes = [P]
    L.tcb_llama_start.argtypes = [P, P, ctypes.c_int, P]
    L.tcb_llama_step.argtypes = [P, P]
    L.tcb_llama_prefill.argtypes = [P, P]
    L.tcb_llama_set_prefill_rows.argtypes = [P, ctypes.c_int]
    L.tcb_llama_prefill_batch.argtypes = [P, ctypes.c_int, P]
    L.tcb_llama_capture.argtypes = [P, P]
    L.tcb_llama_step_kernels.argtypes = [P, ctypes.POINTER(ctypes.c_int)]
    L.tcb_llama_buffers.argtypes = [P, ctypes.POINTER(P), ctypes.POINTER(P)]
    L.tcb_nccl_unique_id.argtypes = [P]
    L.tcb_llama_tp_init.argtypes = [P, P]
    L.tcb_llama_peer_handle.argtypes = [P, P]
    L.tcb_llama_peer_init.argtypes = [P, P]
    L.tcb_llama_batch_create.argtypes = [P, ctypes.c_int, ctypes.POINTER(P)]
    L.tcb_llama_batch_destroy.argtypes = [P]
    L.tcb_llama_batch_step.argtypes = [P, P]
    L.tcb_llama_batch_capture.argtypes = [P, P]
    L.tcb_llama_batch_logits.argtypes = [P, ctypes.POINTER(P)]
    L._llama_bound = True
    return L


class Llama:
    """A decoder engine over a device model (keeps the model alive)."""

    def __init__(self, ctx, model: dict, tp: tuple = (1, 0)):
        """model: this rank's tensors (device_model(..., tp=tp)); tp = (size, rank)."""
        L = _bind()
        cfg = model["cfg"]
        self.cfg, self.model, self._L, self.tp = cfg, model, L, tp
        c = _Cfg(cfg.n_layers, cfg.d_model, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn_dim, cfg.vocab,
                 cfg.max_ctx, cfg.eps, cfg.rope_theta, tp[0], tp[1])

        def arr(ts):
            return (ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts])

        self._arrs = {k: arr(model[k]) for k in ("attn_norm", "ffn_norm", "qkv", "o", "gate_up", "down")}
        types = model.get("types") or {}
        self._lt = None
        if any(k in types for k in LAYER_KINDS):
            flat = [t for row in layer_types(model) for t in row]
            self._lt = (ctypes.c_int * len(flat))(*flat)
        w = _Weights(model["tok_emb"].data_ptr(), types.get("tok_emb", TYPES["tok_emb"]), model["final_norm"].data_ptr(),
                     model["head"].data_ptr(), types.get("head", TYPES["head"]),
                     ctypes.cast(self._arrs["attn_norm"], _PP), ctypes.cast(self._arrs["ffn_norm"], _PP),
                     ctypes.cast(self._arrs["qkv"], _PP), TYPES["qkv"], ctypes.cast(self._arrs["o"], _PP),
                     TYPES["o"], ctypes.cast(self._arrs["gate_up"], _PP), TYPES["gate_up"],
                     ctypes.cast(self._arrs["down"], _PP), TYPES["down"],
                     ctypes.cast(self._lt, ctypes.POINTER(ctypes.c_int)) if self._lt is not None else None)
        h = ctypes.c_void_p()
        self._check(L.tcb_llama_create(ctx.handle, ctypes.byref(c), ctypes.byref(w), ctypes.byref(h)), "create")
        self._h = h
        self._ctx = ctx

    def _check(self, rc, what):
        if rc != 0:
            err = TcbError(rc, f"tcb_llama_{what}")
            if rc == 5:
                err.args = (err.args[0] + ": " + self._L.tcb_last_cuda_error(self._ctx.handle).decode(),)
            raise err

    def start(self, prompt, stream=None):
        p = np.ascontiguousarray(prompt, dtype=np.int64)
        self._check(self._L.tcb_llama_start(self._h, p.ctypes.data, p.size, _stream(stream)), "start")

    def set_prefill_rows(self, rows: int):
        """Rows per pass of prefill (0: the default 2048)."""
        self._check(self._L.tcb_llama_set_prefill_rows(self._h, rows), "set_prefill_rows")

    def prefill(self, stream=None):
        """Feed all but the last prompt token in row batches (directly after
        start); the next step feeds the last one and takes the first greedy
        token."""
        self._check(self._L.tcb_llama_prefill(self._h, _stream(stream)), "prefill")

    def step(self, n: int = 1, stream=None):
        s = _stream(stream)
        for _ in range(n):
            self._check(self._L.tcb_llama_step(self._h, s), "step")

    def capture(self, stream=None):
        self._check(self._L.tcb_llama_capture(self._h, _stream(stream)), "capture")

    def step_kernels(self) -> int:
        """Kernel launches in one captured step (after capture)."""
        n = ctypes.c_int(0)
        self._check(self._L.tcb_llama_step_kernels(self._h, ctypes.byref(n)), "step_kernels")
        return n.value

    def _buffers(self):
        t, lg = ctypes.c_void_p(), ctypes.c_void_p()
        self._check(self._L.tcb_llama_buffers(self._h, ctypes.byref(t), ctypes.byref(lg)), "buffers")
        return t.value, lg.value

    def _download(self, ptr: int, out: np.ndarray, stream=None) -> np.ndarray:
        rc = self._L.tcb_quant_download(self._ctx.handle, ptr, out.nbytes, out.ctypes.data, _stream(stream))
        self._check(rc, "download")
        return out

    def tokens(self, n: int, stream=None) -> np.ndarray:
        """The first n entries of the token history (prompt, then greedy)."""
        return self._download(self._buffers()[0], np.empty(n, np.int64), stream)

    def logits(self, stream=None) -> np.ndarray:
        """The logits of the last step (this rank's vocabulary rows)."""
        n = self.cfg.vocab // self.tp[0]
        return self._download(self._buffers()[1], np.empty(n, np.float32), stream)

    def tp_init(self, nccl_id: bytes, peer: bool = True):
        """Join the tensor-parallel group (every rank, the same 128-byte id).
        With peer=True the residual all-reduce runs over NVLink peer memory:
        the ranks' CUDA IPC handles are gathered in rank order over the
        default torch.distributed group (every rank must call this).  If the
        peers cannot be mapped the step keeps NCCL's all-reduce
        (self.peer_active says which)."""
        buf = ctypes.create_string_buffer(bytes(nccl_id), 128)
        self._check(self._L.tcb_llama_tp_init(self._h, buf), "tp_init")
        self.peer_active = False
        if not peer or self.tp[0] == 1:
            return
        h = ctypes.create_string_buffer(64)
        ok = self._L.tcb_llama_peer_handle(self._h, h) == 0
        handles = gather_bytes(h.raw if ok else b"", self.tp[0])
        if ok and all(len(x) == 64 for x in handles):
            hb = ctypes.create_string_buffer(b"".join(handles), 64 * len(handles))
            ok = self._L.tcb_llama_peer_init(self._h, hb) == 0
        else:
            ok = False
        # every rank takes the same path: peer only if all ranks mapped their peers
        self.peer_active = all(gather_bytes(b"1" if ok else b"0", self.tp[0])[i] == b"1" for i in range(self.tp[0]))
        if ok and not self.peer_active:
            raise RuntimeError("peer all-reduce set up on some ranks only")

    def close(self):
        if getattr(self, "_h", None):
            self._L.tcb_llama_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Batch:
    """Greedy decode of several engines on the same model together
    (tcb_llama_batch_*): each step feeds every sequence its current token,
    the products run once over all of them.  Keeps the engines alive."""

    def __init__(self, engines: list):
        self.engines = list(engines)
        e0 = self.engines[0]
        self._L, self.cfg, self.tp = e0._L, e0.cfg, e0.tp
        arr = (ctypes.c_void_p * len(engines))(*[e._h.value for e in engines])
        h = ctypes.c_void_p()
        e0._check(self._L.tcb_llama_batch_create(arr, len(engines), ctypes.byref(h)), "batch_create")
        self._h = h

    def step(self, n: int = 1, stream=None):
        s = _stream(stream)
        for _ in range(n):
            self.engines[0]._check(self._L.tcb_llama_batch_step(self._h, s), "batch_step")

    def capture(self, stream=None):
        self.engines[0]._check(self._L.tcb_llama_batch_capture(self._h, _stream(stream)), "batch_capture")

    def logits(self, stream=None) -> np.ndarray:
        """[count, vocab] logits of the last step (this rank's vocabulary rows)."""
        p = ctypes.c_void_p()
        self.engines[0]._check(self._L.tcb_llama_batch_logits(self._h, ctypes.byref(p)), "batch_logits")
        n = self.cfg.vocab // self.tp[0]
        return self.engines[0]._download(p.value, np.empty((len(self.engines), n), np.float32), stream)

    def close(self):
        if getattr(self, "_h", None):
            self._L.tcb_llama_batch_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def prefill_batch(engines: list, stream=None):
    """The prompt pass of several engines on the same model at once (each
    started with its own prompt): one set of rows through the products."""
    if not engines:
        return
    arr = (ctypes.c_void_p * len(engines))(*[e._h.value for e in engines])
    engines[0]._check(engines[0]._L.tcb_llama_prefill_batch(arr, len(engines), _stream(stream)), "prefill_batch")


def nccl_unique_id() -> bytes:
    """A fresh NCCL id (rank 0 makes it, every rank passes it to tp_init)."""
    L = _bind()
    buf = ctypes.create_string_buffer(128)
    rc = L.tcb_nccl_unique_id(buf)
    if rc != 0:
        raise TcbError(rc, "tcb_nccl_unique_id")
    return buf.raw


def gather_bytes(b: bytes, world: int) -> list:
    """Every rank's bytes, in rank order, on every rank of the default
    torch.distributed group (any backend)."""
    import torch.distributed as dist

    out = [None] * world
    dist.all_gather_object(out, bytes(b))
    return out


def share_id(make, rank: int) -> bytes:
    """Rank 0's make() result on every rank of the default torch.distributed
    group (any backend)."""
    import torch.distributed as dist

    obj = [make() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    return obj[0]
