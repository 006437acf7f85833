"""The native GGUF reader (bebelm_gguf_*) against the reference's own GGUF tests
(src/gguf.rs:434-659, src/config.rs:109-233) and against the CPU restatement
``oracle/gguf.py`` on seeded random files, truncations and byte flips. CPU only, except the
last test, which uploads an attention layer and the logits head from a file."""
import random
import struct

import numpy as np
import pytest

import bebelm_b200 as bb
import gguf_build as gb
from oracle import gguf as og


def sample() -> bytes:
    """build_sample (src/gguf.rs:443-490): 3 kvs, tensors a [4] F32 at 0 and b [2,3] F32 at 16."""
    buf = b"GGUF" + struct.pack("<IQQ", 3, 2, 3)
    buf += gb.kv("general.architecture", gb.STRING, "lfm2_moe")
    buf += gb.kv("lfm2_moe.block_count", gb.U32, 24)
    buf += gb.kv("tokenizer.ggml.tokens", gb.ARRAY, (gb.STRING, ["<bos>", "hello"]))
    buf += gb.tensor_entry("a", [4], 0, 0) + gb.tensor_entry("b", [2, 3], 0, 16)
    buf += b"\0" * (-len(buf) % 32)
    buf += struct.pack("<4f", 1, 2, 3, 4) + struct.pack("<6f", 10, 11, 12, 13, 14, 15)
    return buf


def header(n_tensors, n_kv, body) -> bytes:
    """header (src/gguf.rs:550-561)."""
    buf = b"GGUF" + struct.pack("<IQQ", 3, n_tensors, n_kv) + body
    return buf + b"\0" * (-len(buf) % 32)


def fmt_err(data) -> str:
    with pytest.raises(bb.BebelmError) as e:
        bb.Gguf(data=data)
    assert e.value.code == bb.ERR_FORMAT
    return str(e.value)


# ------------------------------------------------------- the reference's tests --
def test_parses_header_and_metadata():
    g = bb.Gguf(data=sample())
    assert g.version == 3 and g.alignment == 32
    assert g.architecture() == "lfm2_moe"
    assert g.get_u32("lfm2_moe.block_count") == 24
    assert g.get_str_array("tokenizer.ggml.tokens") == ["<bos>", "hello"]


def test_parses_tensors_and_data():
    g = bb.Gguf(data=sample())
    a, b = g.tensors
    assert (a["name"], a["dims"], a["ggml_type"], a["n_elements"], a["data_len"]) == ("a", [4], 0, 4, 16)
    assert (b["name"], b["dims"], b["n_elements"]) == ("b", [2, 3], 6)
    assert np.frombuffer(g.tensor_data("a"), np.float32).tolist() == [1, 2, 3, 4]
    assert np.frombuffer(g.tensor_data("b"), np.float32)[0] == 10.0


def test_rejects_bad_magic():
    buf = bytearray(sample())
    buf[0] = ord("X")
    assert "not a GGUF file" in fmt_err(bytes(buf))


def test_rejects_truncated_file():
    assert "unexpected end of file" in fmt_err(sample()[:10])


def test_rejects_unsupported_version():
    buf = bytearray(sample())
    buf[4:8] = struct.pack("<I", 5)
    assert "unsupported GGUF version 5" in fmt_err(bytes(buf))


def test_rejects_unknown_value_type():
    body = gb.gstr("weird") + struct.pack("<I", 99)
    assert "unknown metadata value type 99" in fmt_err(header(0, 1, body))


def test_rejects_unknown_tensor_type():
    body = gb.tensor_entry("weird", [1], 1000, 0)
    assert "unmodeled ggml type 1000" in fmt_err(header(1, 0, body))


def test_rejects_tensor_out_of_bounds():
    body = gb.tensor_entry("big", [1024], 0, 0)
    assert "outside the file" in fmt_err(header(1, 0, body))


def test_reads_custom_alignment():
    g = bb.Gguf(data=header(0, 1, gb.kv("general.alignment", gb.U32, 8)))
    assert g.alignment == 8


def test_accessors_widen_integer_and_float_types():
    body = (gb.kv("k.u8", gb.U8, 7) + gb.kv("k.i64", gb.I64, 123) + gb.kv("k.f64", gb.F64, 2.5) +
            gb.kv("k.i16arr", gb.ARRAY, (gb.I16, [10, 0, 8])))
    g = bb.Gguf(data=header(0, 4, body))
    assert g.get_u32("k.u8") == 7 and g.get_u32("k.i64") == 123
    assert g.get_f32("k.f64") == 2.5
    assert g.get_u32_array("k.i16arr") == [10, 0, 8]
    assert g.get_u32("missing") is None and g.get_f32("k.u8") is None and g.get_str("k.u8") is None


def test_rejects_invalid_utf8():
    body = struct.pack("<Q", 2) + b"\xc3\x28" + struct.pack("<I", gb.U8) + b"\x01"
    assert "invalid UTF-8" in fmt_err(header(0, 1, body))


def test_validate_accepts_matching_metadata():
    bb.Gguf(data=gb.build(gb.model_kvs())).validate()


@pytest.mark.parametrize("kvs,what", [(gb.model_kvs(arch="llama"), "architecture"),
                                      (gb.model_kvs(block_count=12), "block_count"),
                                      (gb.model_kvs(schedule=[0] * 24), "schedule mismatch")])
def test_validate_rejects(kvs, what):
    with pytest.raises(bb.BebelmError) as e:
        bb.Gguf(data=gb.build(kvs)).validate()
    assert e.value.code == bb.ERR_FORMAT and what in str(e.value)


def test_open_maps_a_file(tmp_path):
    p = tmp_path / "m.gguf"
    p.write_bytes(sample())
    g = bb.Gguf(str(p))

    def strip(ts):
        return [{k: v for k, v in t.items() if k != "data_ptr"} for t in ts]

    assert strip(g.tensors) == strip(bb.Gguf(data=sample()).tensors)
    assert np.frombuffer(g.tensor_data("a"), np.float32).tolist() == [1, 2, 3, 4]
    with pytest.raises(bb.BebelmError) as e:
        bb.Gguf(str(tmp_path / "absent.gguf"))
    assert e.value.code == bb.ERR_IO


# ------------------------------------------------- against the CPU restatement --
_SCALARS = [gb.U8, gb.I8, gb.U16, gb.I16, gb.U32, gb.I32, gb.F32, gb.BOOL, gb.STRING, gb.U64, gb.I64, gb.F64]
_INTS = (gb.U8, gb.I8, gb.U16, gb.I16, gb.U32, gb.I32, gb.U64, gb.I64)


def _rand_value(rng, vt, depth=0):
    if vt == gb.STRING:
        return "".join(rng.choice("abcé€𝄞_.") for _ in range(rng.randint(0, 6)))
    if vt == gb.ARRAY:
        et = rng.choice(_SCALARS + ([gb.ARRAY] if depth < 2 else []))
        return et, [_rand_value(rng, et, depth + 1) for _ in range(rng.randint(0, 4))]
    if vt in (gb.F32, gb.F64):
        return float(np.float32(rng.uniform(-1e6, 1e6))) if vt == gb.F32 else rng.uniform(-1e300, 1e300)
    if vt == gb.BOOL:
        return rng.randint(0, 1)
    bits = {gb.U8: 8, gb.I8: 8, gb.U16: 16, gb.I16: 16, gb.U32: 32, gb.I32: 32, gb.U64: 64, gb.I64: 64}[vt]
    if vt in (gb.I8, gb.I16, gb.I32, gb.I64):
        return rng.randint(-(1 << (bits - 1)), (1 << (bits - 1)) - 1)
    return rng.randint(0, (1 << bits) - 1)


def _rand_file(rng) -> bytes:
    kvs = []
    for k in range(rng.randint(0, 8)):
        vt = rng.choice(_SCALARS + [gb.ARRAY])
        kvs.append((f"key.{k % 6}", vt, _rand_value(rng, vt)))  # repeated keys: the last one wins
    if rng.random() < 0.3:
        kvs.append(("general.alignment", rng.choice([gb.U32, gb.U64, gb.U16]), rng.choice([1, 8, 16, 32, 64])))
    tensors = []
    for t in range(rng.randint(0, 5)):
        ty = rng.choice([0, 1, 12, 14, 8, 30])
        be, bb_ = og.BLOCKS[ty]
        dims = [be * rng.randint(1, 3)] + [rng.randint(1, 3) for _ in range(rng.randint(0, 2))]
        n = int(np.prod(dims))
        tensors.append((f"t{t}", dims, ty, bytes(rng.getrandbits(8) for _ in range(n // be * bb_))))
    al = [v for k, _, v in kvs if k == "general.alignment"]
    return gb.build(kvs, tensors, alignment=32 if not al else 64, version=rng.choice([2, 3]))


_WORDS = {"BadMagic": "not a GGUF file", "UnsupportedVersion": "unsupported GGUF version",
          "UnexpectedEof": "unexpected end of file", "UnknownValueType": "unknown metadata value type",
          "InvalidUtf8": "invalid UTF-8", "UnknownTensorType": "unmodeled ggml type",
          "TensorOutOfBounds": "outside the file"}


def _compare(data: bytes) -> bool:
    """Parses `data` both ways; the same verdict, and on success the same contents."""
    try:
        want = og.parse(data)
    except og.GgufError as e:
        msg = fmt_err(data)
        assert _WORDS[e.kind] in msg, (e.kind, msg)
        return False
    g = bb.Gguf(data=data)
    assert (g.version, g.alignment, g.data_offset) == (want["version"], want["alignment"], want["data_offset"])
    assert [k for k, _ in g.keys()] == list(want["metadata"])
    for (k, vt), (wt, wv) in zip(g.keys(), want["metadata"].values()):
        assert vt == wt, k
        if "\0" in k:
            continue  # the typed lookups take NUL-terminated keys
        if wt in _INTS:
            assert g.get_u32(k) == wv & 0xFFFFFFFF, k
        elif wt in (gb.F32, gb.F64):
            with np.errstate(over="ignore"):
                assert np.float32(g.get_f32(k)).tobytes() == np.float32(wv).tobytes(), k
        elif wt == gb.STRING:
            assert g.get_str(k) == wv, k
        elif wt == gb.ARRAY:
            et, items = wv
            if et == gb.STRING:
                assert g.get_str_array(k) == items, k
            elif et in _INTS:
                assert g.get_u32_array(k) == [x & 0xFFFFFFFF for x in items], k
    got = [{k: t[k] for k in ("name", "dims", "n_dims", "ggml_type", "offset", "data_start", "data_len",
                              "n_elements")} for t in g.tensors]
    assert got == [dict(t, dims=t["dims"][:8], n_dims=len(t["dims"])) for t in want["tensors"]]
    for t in want["tensors"]:
        if "\0" not in t["name"]:
            assert g.tensor_data(t["name"]) == data[t["data_start"]:t["data_start"] + t["data_len"]]
    return True


def test_random_files_match_restatement():
    rng = random.Random(1234)
    ok = sum(_compare(_rand_file(rng)) for _ in range(300))
    assert ok > 200


def test_truncations_and_flips_match_restatement():
    rng = random.Random(99)
    for _ in range(200):
        data = _rand_file(rng)
        for cut in sorted(set(rng.randrange(0, len(data) + 1) for _ in range(4))):
            _compare(data[:cut])
        for _ in range(8):
            b = bytearray(data)
            b[rng.randrange(0, len(b))] = rng.getrandbits(8)
            _compare(bytes(b))


# ---------------------------------------------------------- uploads from a file --
def _kquant(rng, rows, n_in, six=False):
    """Random K-quant rows with sane f16 scales (as the projection tests use)."""
    bb_ = 210 if six else 144
    w = rng.integers(0, 256, size=(rows, n_in // 256, bb_), dtype=np.uint8)
    d = (rng.standard_normal((rows, n_in // 256)) * (0.002 if six else 0.01)).astype(np.float16)
    w[:, :, (208 if six else 0):(210 if six else 2)] = d.view(np.uint8).reshape(rows, -1, 2)
    if not six:
        w[:, :, 2:4] = (np.abs(rng.standard_normal((rows, n_in // 256))) * 0.005).astype(
            np.float16).view(np.uint8).reshape(rows, -1, 2)
    return w.reshape(-1)


@pytest.mark.gpu
def test_layer_and_head_from_a_gguf_file(tmp_path):
    """A synthetic model file (the reference's metadata and tensor names, random weights):
    the attention layer and the head uploaded from it compute exactly what the same bytes
    uploaded directly compute."""
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(3)
    H, KV, HID, VOCAB = 32, 8, 2048, 3000
    wq, wk = _kquant(rng, H * 64, HID), _kquant(rng, KV * 64, HID)
    wv, wo = _kquant(rng, KV * 64, HID, six=True), _kquant(rng, HID, H * 64)
    qg = (1 + 0.02 * rng.standard_normal(64)).astype(np.float32)
    kg = (1 + 0.02 * rng.standard_normal(64)).astype(np.float32)
    te = _kquant(rng, VOCAB, HID, six=True)
    ng = (1 + 0.02 * rng.standard_normal(HID)).astype(np.float32)
    tensors = [("token_embd.weight", [HID, VOCAB], 14, te.tobytes()),
               ("token_embd_norm.weight", [HID], 0, ng.tobytes()),
               ("blk.2.attn_q.weight", [HID, H * 64], 12, wq.tobytes()),
               ("blk.2.attn_k.weight", [HID, KV * 64], 12, wk.tobytes()),
               ("blk.2.attn_v.weight", [HID, KV * 64], 14, wv.tobytes()),
               ("blk.2.attn_output.weight", [H * 64, HID], 12, wo.tobytes()),
               ("blk.2.attn_q_norm.weight", [64], 0, qg.tobytes()),
               ("blk.2.attn_k_norm.weight", [64], 0, kg.tobytes())]
    p = tmp_path / "model.gguf"
    p.write_bytes(gb.build(gb.model_kvs(), tensors))
    g = bb.Gguf(str(p))
    g.validate()
    Wf = g.attn_weights(2)
    Wd = bb.AttnWeights((12, wq), (12, wk), (14, wv), (12, wo), qg, kg)
    with pytest.raises(bb.BebelmError) as e:
        g.attn_weights(3)  # a short-conv block has no attention tensors
    assert e.value.code == bb.ERR_NOT_FOUND
    x = torch.from_numpy((0.5 * rng.standard_normal((40, HID))).astype(np.float32)).cuda()
    outs = []
    for W in (Wf, Wd):
        c = bb.Cache(n_layers=1, max_context=256)
        o = torch.empty((40, HID), device="cuda")
        bb.attn_layer_batch(c, 0, W, x[:32], 0, tensor_cores=False, theta=5e6, out=o[:32])
        for i in range(32, 40):
            bb.attn_layer_step(c, 0, W, x[i], i, theta=5e6, out=o[i])
        torch.cuda.synchronize()
        outs.append(o.cpu().numpy())
        c.close()
    assert np.array_equal(outs[0], outs[1])
    hf = g.head()
    hd = bb.Head(14, te, HID, VOCAB, ng)
    h = rng.standard_normal(HID).astype(np.float32)
    lf, tf = hf.logits(h)
    ld, td = hd.logits(h)
    assert np.array_equal(lf, ld) and tf == td
    for o in (Wf, Wd, hf, hd, g):
        o.close()
