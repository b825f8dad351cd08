"""GGUF v3 header decoding and the llama file mapping, on the CPU.

Mirrors TR's gguf tests (internal/compute/gguf/gguf_test.go): malformed
headers are rejected with the kind of failure (TestDecodeRejects), every
truncation of a valid file is an error (TestDecodeTruncatedEverywhere), the
decoder never reads past the stated size (TestDecodeHoldsToSize), every known
tensor type is accepted (TestDecodeAcceptsEveryKnownType); plus the llama
mapping's round trip (names, q/k row order, merged qkv and gate/up rows)."""
import struct

import numpy as np
import pytest

from tcb_b200 import gguf as G


def small_file(**kw):
    b = G.Builder(**kw)
    b.kv("general.architecture", "llama").kv("n", (G.U32, 7)).kv("f", 0.5).kv("flag", True)
    b.kv("names", ["a", "bc", ""]).kv("ids", [(G.I32, 1), (G.I32, -2)])
    b.tensor("w", G.Q4_K, [512, 2], bytes(range(256)) * 2 + bytes(576 - 512))
    b.tensor("n", G.F32, [5], np.arange(5, dtype=np.float32).tobytes())
    return b.to_bytes()


def header(version=3, tensors=0, keys=0):
    return G.MAGIC + struct.pack("<IQQ", version, tensors, keys)


def kv(key, vt, body):
    k = key.encode()
    return struct.pack("<Q", len(k)) + k + struct.pack("<I", vt) + body


def tensor_rec(name, dims, ttype, offset):
    n = name.encode()
    out = struct.pack("<Q", len(n)) + n + struct.pack("<I", len(dims))
    return out + b"".join(struct.pack("<Q", d) for d in dims) + struct.pack("<IQ", ttype, offset)


def kind_of(data, size=None):
    with pytest.raises(G.GGUFError) as e:
        G.decode(data, size)
    return e.value.kind


def test_round_trip_values_and_tensors():
    data = small_file()
    f = G.decode(data)
    assert f.keys == ["general.architecture", "n", "f", "flag", "names", "ids"]
    assert f.values["n"].type == G.U32 and f.values["n"].data == 7
    assert f.values["f"].data == 0.5 and f.values["flag"].data is True
    assert f.values["names"].data == ["a", "bc", ""] and f.values["names"].elem == G.STRING
    assert f.values["ids"].data == [1, -2]
    w, n = f.tensors
    assert (w.dims, w.size, w.offset, w.shape()) == ([512, 2], 576, 0, (2, 512))
    assert (n.size, n.offset) == (20, 576)
    assert f.data_start % 32 == 0 and f.data_start >= f.header_end
    assert bytes(G.tensor_bytes(data, f, w))[:256] == bytes(range(256))
    assert np.array_equal(np.frombuffer(G.tensor_bytes(data, f, n), np.float32), np.arange(5))


def test_custom_alignment():
    data = small_file(alignment=64)
    f = G.decode(data)
    assert f.alignment == 64 and f.data_start % 64 == 0 and f.tensors[1].offset == 576


def test_truncated_everywhere():
    data = small_file()
    for n in range(len(data)):
        assert kind_of(data, n) in ("truncated", "length", "counts", "range"), n
    G.decode(data)


def test_holds_to_size():
    """An array declared far longer than the file fails on its length, at
    every stated size; a stream longer than the size is not read past it."""
    body = struct.pack("<IQ", G.U8, 1 << 50)
    data = header(3, 0, 1) + kv("k", G.ARRAY, body) + bytes(1 << 10)
    assert kind_of(data, 0) == "truncated"
    assert kind_of(data, 10) == "truncated"
    assert kind_of(data, len(data) - (1 << 10) - 4) == "truncated"
    assert kind_of(data, len(data) - (1 << 10)) == "length"
    assert kind_of(data) == "length"
    good = small_file()
    assert kind_of(good + bytes(100), len(good) - 1) in ("truncated", "range")


@pytest.mark.parametrize("case,kind", [
    (b"GGUG" + struct.pack("<IQQ", 3, 0, 0), "magic"),
    (header(version=2), "version"),
    (header(version=0x03000000), "version"),
    (header(3, 1 << 40, 0), "counts"),
    (header(3, 0, 1 << 60), "counts"),
    (header(3, 0, 1) + kv("k", 13, b"\0" * 8), "value_type"),
    (header(3, 0, 1) + kv("k", G.ARRAY, struct.pack("<IQ", G.ARRAY, 0)), "nested"),
    (header(3, 0, 1) + kv("k", G.ARRAY, struct.pack("<IQ", 99, 0)), "value_type"),
    (header(3, 0, 1) + kv("k", G.BOOL, b"\x02"), "bool"),
    (header(3, 0, 1) + kv("k", G.STRING, struct.pack("<Q", 2) + b"\xff\xfe"), "utf8"),
    (header(3, 0, 2) + kv("k", G.U8, b"\1") + kv("k", G.U8, b"\1"), "duplicate"),
    (header(3, 0, 1) + kv("general.alignment", G.U32, struct.pack("<I", 48)), "alignment"),
    (header(3, 0, 1) + kv("general.alignment", G.U64, struct.pack("<Q", 64)), "alignment"),
    (header(3, 1, 0) + tensor_rec("x" * 64, [32], G.F32, 0) + bytes(256), "name"),
    (header(3, 1, 0) + tensor_rec("", [32], G.F32, 0) + bytes(256), "name"),
    (header(3, 1, 0) + tensor_rec("t", [1, 1, 1, 1, 1], G.F32, 0) + bytes(256), "dims"),
    (header(3, 1, 0) + tensor_rec("t", [1 << 63], G.F32, 0) + bytes(256), "dim"),
    (header(3, 1, 0) + tensor_rec("t", [32], 5, 0) + bytes(256), "type"),
    (header(3, 1, 0) + tensor_rec("t", [100], G.Q4_K, 0) + bytes(256), "block"),
    (header(3, 1, 0) + tensor_rec("t", [1 << 40, 1 << 40], G.F32, 0) + bytes(256), "size"),
    (header(3, 2, 0) + tensor_rec("t", [8], G.F32, 0) + tensor_rec("t", [8], G.F32, 32) + bytes(256), "duplicate"),
    (header(3, 1, 0) + tensor_rec("t", [8], G.F32, 32) + bytes(256), "offset"),
    (header(3, 1, 0) + tensor_rec("t", [1024], G.F32, 0) + bytes(64), "range"),
])
def test_rejects(case, kind):
    assert kind_of(case) == kind


def test_accepts_every_known_type():
    b = G.Builder()
    for t, (name, blk, bb) in G.TYPES.items():
        b.tensor(f"t{t}", t, [blk * 2], bytes(2 * bb))
    f = G.decode(b.to_bytes())
    assert [t.type for t in f.tensors] == list(G.TYPES)
    assert all(t.size == 2 * G.TYPES[t.type][2] for t in f.tensors)


def test_llama_round_trip(tmp_path):
    from tcb_b200 import llama, llama_gguf

    cfg = llama.LlamaConfig(n_layers=2, d_model=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn_dim=1024,
                            vocab=2048, max_ctx=160)
    host = llama.host_model(cfg, seed=3)
    path = str(tmp_path / "tiny.gguf")
    llama_gguf.write(path, cfg, host)
    f = G.decode(open(path, "rb").read())
    names = [t.name for t in f.tensors]
    assert names[0] == "token_embd.weight" and names[-2:] == ["output_norm.weight", "output.weight"]
    assert "blk.1.ffn_down.weight" in names and f.values["llama.block_count"].data == 2
    # the file's attn_q rows are in the converter's interleaved order
    q = np.frombuffer(G.tensor_bytes(open(path, "rb").read(), f, f.tensor("blk.0.attn_q.weight")), np.uint8)
    rows = host["qkv"][0].reshape((4 + 2 * 2) * 128, -1)
    frow = q.reshape(4 * 128, -1)
    assert np.array_equal(frow[2], rows[1]) and np.array_equal(frow[1], rows[64]) and np.array_equal(frow[129], rows[192])
    cfg2, host2 = llama_gguf.load(path)
    # eps and rope_theta are stored as F32 metadata (the engine takes them as float32)
    assert cfg2.eps == float(np.float32(cfg.eps)) and cfg2.rope_theta == float(np.float32(cfg.rope_theta))
    assert cfg2.__class__(**{**cfg2.__dict__, "eps": cfg.eps, "rope_theta": cfg.rope_theta}) == cfg
    for k in ("tok_emb", "head", "final_norm"):
        assert np.array_equal(np.asarray(host2[k]), np.asarray(host[k])), k
    for k in ("attn_norm", "ffn_norm", "qkv", "o", "gate_up", "down"):
        for a, b in zip(host2[k], host[k]):
            assert np.array_equal(np.asarray(a), np.asarray(b)), k


def test_llama_load_rejects(tmp_path):
    from tcb_b200 import TcbError, llama, llama_gguf

    cfg = llama.LlamaConfig(n_layers=1, d_model=256, n_heads=2, n_kv_heads=1, head_dim=128, ffn_dim=256,
                            vocab=256, max_ctx=64)
    host = llama.host_model(cfg, seed=4)
    bad = dict(host)
    bad["down"] = [host["down"][0].copy()]
    bad["down"][0][208:210] = np.array([0x00, 0x7C], np.uint8)  # +Inf fp16 scale in block 0
    path = str(tmp_path / "bad.gguf")
    llama_gguf.write(path, cfg, bad)
    with pytest.raises(TcbError):
        llama_gguf.load(path)
    path2 = str(tmp_path / "arch.gguf")
    b = G.Builder().kv("general.architecture", "gemma3")
    b.write(path2)
    with pytest.raises(ValueError):
        llama_gguf.load(path2)


def test_llama_round_trip_mixed_types(tmp_path):
    """llama.cpp Q4_K_M-like files: attn_v and ffn_down Q6_K in some layers
    and Q4_K in others, a Q4_0 head and a Q8_0 output projection in one
    layer: every tensor keeps its own type and bytes through write and load;
    q/k (or gate/up) of different types are refused (one merged product)."""
    import tcb_b200 as T
    from tcb_b200 import llama, llama_gguf

    cfg = llama.LlamaConfig(n_layers=3, d_model=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn_dim=1024,
                            vocab=2048, max_ctx=160)
    types = {"v": [T.Q6_K, T.Q4_K, T.Q6_K], "down": [T.Q6_K, T.Q4_K, T.Q4_K], "o": [T.Q6_K, T.Q8_0, T.Q6_K]}
    host = llama.host_model(cfg, seed=5, types=types)
    path = str(tmp_path / "mixed.gguf")
    llama_gguf.write(path, cfg, host)
    f = G.decode(open(path, "rb").read())
    assert f.tensor("blk.0.attn_v.weight").type == T.Q6_K and f.tensor("blk.1.attn_v.weight").type == T.Q4_K
    assert f.tensor("blk.1.attn_output.weight").type == T.Q8_0
    assert f.tensor("blk.1.ffn_down.weight").type == T.Q4_K
    cfg2, host2 = llama_gguf.load(path)
    assert host2["types"] == types
    for k in ("qkv", "o", "gate_up", "down"):
        for a, b in zip(host2[k], host[k]):
            assert np.array_equal(np.asarray(a), np.asarray(b)), k
    assert llama.layer_types(host2) == llama.layer_types(host)
    # q and k of different types cannot be merged
    b = G.Builder()
    for k, v in f.values.items():
        b.kv(k, v.data if isinstance(v.data, str) else (v.type, v.data))
    raw = open(path, "rb").read()
    for t in f.tensors:
        data = G.tensor_bytes(raw, f, t)
        if t.name == "blk.2.attn_k.weight":
            # the same rows re-encoded as Q8_0 blocks of zeros: a type the q rows do not share
            data = np.zeros(t.dims[1] * t.dims[0] // 32 * 34, np.uint8).tobytes()
            b.tensor(t.name, T.Q8_0, list(t.dims), data)
        else:
            b.tensor(t.name, t.type, list(t.dims), data)
    path2 = str(tmp_path / "qk.gguf")
    b.write(path2)
    with pytest.raises(ValueError, match="attn_q and attn_k"):
        llama_gguf.load(path2)
