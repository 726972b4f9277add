"""CPU: the GGUF tensor index (bread_gguf_*), the loader front end of row f2
(gguf.c:306-411 parsing; loader.c:156-206 tensor names and expert ranges).

Fixtures are written by tests/gguf_file.py.  The parser is checked against
the reference's own gguf_open compiled in oracle/_ref (same tensor infos and
data offset on the same file), and must refuse malformed files with a status
instead of exiting the process as the reference does."""
import os

import numpy as np
import pytest

import breadv2_b200 as bb
import gguf_file as G

Q4_K, Q6_K = 12, 14


def _fixture(path, alignment=None):
    rng = np.random.default_rng(1)
    ts = [("blk.0.ffn_gate_exps.weight", Q4_K, [512, 256, 4], rng.integers(0, 256, 4 * 256 * 2 * 144, np.uint8)),
          ("blk.0.ffn_gate_inp.weight", 0, [512, 4], rng.standard_normal(2048).astype(np.float32)),
          ("blk.0.ffn_gate_inp_shexp.weight", 1, [512], rng.standard_normal(512).astype(np.float16)),
          ("blk.0.ffn_down_exps.weight", Q6_K, [256, 512, 4], rng.integers(0, 256, 4 * 512 * 210, np.uint8)),
          ("output.weight", 8, [512, 7], rng.integers(0, 256, 7 * 16 * 34, np.uint8))]
    kv = [("general.architecture", G.STR, "qwen35moe"), ("general.name", G.STR, "fixture"),
          ("a.u8", G.U8, 7), ("a.i16", G.I16, -3), ("a.f32", G.F32, 1.5), ("a.bool", G.BOOL, True),
          ("a.u64", G.U64, 1 << 40), ("a.f64", G.F64, 2.25),
          ("tokenizer.ggml.tokens", G.ARR, (G.STR, ["<s>", "hello", "wörld"] * 50)),
          ("tokenizer.ggml.scores", G.ARR, (G.F32, [0.5] * 300)),
          ("nested", G.ARR, (G.ARR, [(G.U16, [1, 2, 3]), (G.STR, ["x"])]))]
    data_off = G.write_gguf(str(path), ts, kv, alignment=alignment)
    return ts, data_off


@pytest.mark.parametrize("alignment", [None, 64, 256])
def test_gguf_index(tmp_path, alignment):
    p = tmp_path / "m.gguf"
    ts, data_off = _fixture(p, alignment)
    g = bb.Gguf(str(p))
    info = g.info()
    assert info == {"version": 3, "n_tensors": len(ts), "alignment": alignment or 32, "data_offset": data_off}
    for i, (name, t, dims, data) in enumerate(ts):
        rec = g.tensor(i)
        assert rec["name"] == name and rec["type"] == t and rec["dims"] == dims
        raw = np.asarray(data).tobytes()
        assert rec["size"] == len(raw) and rec["n_elems"] == int(np.prod(dims))
        assert g.find(name) == rec
        assert g.read(rec["offset"], rec["size"]).tobytes() == raw
    assert g.find("blk.1.ffn_gate_exps.weight") is None
    g.close()


def test_gguf_index_matches_reference_parser(tmp_path, orc):
    """Same file through the reference's gguf_open (compiled from gguf.c)."""
    if not orc.ref_available():
        pytest.skip("reference CPU library not built here")
    p = tmp_path / "m.gguf"
    ts, _ = _fixture(p, 64)
    ref = orc.ref_gguf_index(str(p))
    g = bb.Gguf(str(p))
    assert g.info()["version"] == ref["version"] and g.info()["data_offset"] == ref["data_offset"]
    for i, r in enumerate(ref["tensors"]):
        assert g.tensor(i) == r


def test_gguf_synthetic_model_file(tmp_path, orc):
    """The model-file writer the GPU test uses: expert tensors with experts
    outermost, one contiguous byte range per expert (loader.c:187-199)."""
    p = tmp_path / "model.gguf"
    G.write_synthetic_model(orc, str(p), 2, 512, 256, 8, seed=9)
    g = bb.Gguf(str(p))
    t = g.find("blk.1.ffn_down_exps.weight")
    assert t["dims"] == [256, 512, 8] and t["type"] == Q6_K
    eb = t["size"] // 8
    e5 = g.read(t["offset"] + 5 * eb, eb)
    assert np.array_equal(e5, orc.synth_blocks(512, Q6_K, 9, G.sid(1, 2, 5)))
    assert g.find("blk.0.post_attention_norm.weight")["type"] == 0


def test_gguf_rejects_malformed_files(tmp_path):
    p = tmp_path / "m.gguf"
    _fixture(p)
    raw = p.read_bytes()
    bad = {
        "magic": b"GGUX" + raw[4:],
        "version": raw[:4] + (4).to_bytes(4, "little") + raw[8:],
        "truncated_header": raw[:20],
        "truncated_meta": raw[:200],
        "truncated_data": raw[:-100],
        "empty": b"",
    }
    for what, content in bad.items():
        q = tmp_path / f"{what}.gguf"
        q.write_bytes(content)
        with pytest.raises(bb.BreadError) as ei:
            bb.Gguf(str(q))
        assert ei.value.status == 1, what
    with pytest.raises(bb.BreadError):
        bb.Gguf(str(tmp_path / "missing.gguf"))
