"""The GGUF reader (moearc_x_gguf_*) on files this test writes: metadata, the tensor index,
stacked expert banks sliced along their last dimension, and the refusal of malformed files.

Mirrors the reference's checks on its reader (crates/moearc-model/src/gguf.rs:166-279: counts
bounded by the file size, rank <= 4, power-of-two alignment, every tensor inside the file;
tensors.rs:237-289: whole blocks and an exact tiling per slice) and its mapped-model test
(tests/mapped_model.rs:36-118: every expert slice is where an independent reader finds it).
No GPU is needed: the reader is host code in the library.
"""
import os
import struct

import numpy as np
import pytest

import gguf_writer as W
from moearc_b200.gguf import GgufError, GgufFile, moe_layout

MXFP4, Q4_0, F32 = 39, 2, 0


def rand_bytes(seed, n):
    return np.random.default_rng(seed).integers(0, 256, n, dtype=np.uint8).tobytes()


def model_writer(alignment=None, H=64, I=96, E=4):
    """One gpt-oss-shaped MoE block: MXFP4 gate/up [H, I, E], down [I, H, E], router f32 [H, E]."""
    w = W.GgufWriter(alignment=alignment)
    w.add("general.architecture", W.STRING, "gpt-oss")
    w.add("gpt-oss.expert_count", W.U32, E)
    w.add("gpt-oss.expert_used_count", W.U32, 2)
    w.add("gpt-oss.embedding_length", W.U64, H)
    w.add("gpt-oss.rope.freq_base", W.F32, 150000.0)
    w.add("gpt-oss.attention.layer_norm_rms_epsilon", W.F64, 1e-5)
    w.add("general.signed", W.I32, -7)
    w.add("general.flag", W.BOOL, True)
    w.add("general.small", W.U8, 200)
    w.add("general.tiny", W.I8, -3)
    w.add("general.short", W.U16, 65000)
    w.add("general.sshort", W.I16, -300)
    w.add("general.big", W.I64, 1 << 40)
    w.add("rope.sections", W.ARRAY, (W.I32, [16, 24, 24, 0]))
    w.add("tokenizer.ggml.tokens", W.ARRAY, (W.STRING, [f"t{i}" for i in range(1500)]))
    w.add("tokenizer.ggml.scores", W.ARRAY, (W.F32, [0.5] * 3000))
    banks = {}
    for i, (name, dims) in enumerate((("ffn_gate_exps", (H, I, E)), ("ffn_up_exps", (H, I, E)),
                                      ("ffn_down_exps", (I, H, E)))):
        data = rand_bytes(10 + i, dims[0] * dims[1] * dims[2] // 32 * 17)
        banks[name] = data
        w.add_tensor(f"blk.0.{name}.weight", dims, MXFP4, data)
    router = np.random.default_rng(3).standard_normal((E, H)).astype(np.float32)
    w.add_tensor("blk.0.ffn_gate_inp.weight", (H, E), F32, router.tobytes())
    banks["router"] = router.tobytes()
    q4 = rand_bytes(20, 32 * 3 * 2 // 32 * 18)
    w.add_tensor("blk.0.q4.weight", (32, 3, 2), Q4_0, q4)
    banks["q4"] = q4
    return w, banks


def test_metadata_and_tensor_index_round_trip(tmp_path):
    w, banks = model_writer()
    path = str(tmp_path / "m.gguf")
    data_off, offs = w.write(path)
    with GgufFile(path) as g:
        assert g.version == 3 and g.alignment == 32 and g.n_tensors == 5
        assert g.str("general.architecture") == "gpt-oss"
        assert g.u64("gpt-oss.expert_count") == 4 and g.u64("gpt-oss.embedding_length") == 64
        assert g.u64("general.flag") == 1 and g.u64("general.small") == 200 and g.u64("general.short") == 65000
        assert g.u64("general.big") == 1 << 40
        assert g.f64("gpt-oss.rope.freq_base") == 150000.0
        assert g.f64("gpt-oss.attention.layer_norm_rms_epsilon") == 1e-5
        for key in ("general.signed", "general.tiny", "general.sshort"):  # negative integers
            with pytest.raises(KeyError):
                g.u64(key)
        with pytest.raises(KeyError):
            g.u64("general.architecture")  # a string
        with pytest.raises(KeyError):
            g.str("gpt-oss.expert_count")  # an integer
        with pytest.raises(KeyError):
            g.f64("gpt-oss.expert_count")
        with pytest.raises(KeyError):
            g.u64("no.such.key")
        assert g.u64("no.such.key", default=9) == 9
        ts = g.tensors()
        assert [t.name for t in ts] == ["blk.0.ffn_gate_exps.weight", "blk.0.ffn_up_exps.weight",
                                        "blk.0.ffn_down_exps.weight", "blk.0.ffn_gate_inp.weight", "blk.0.q4.weight"]
        for t, off in zip(ts, offs):
            assert t.offset == data_off + off and t.offset % 32 == 0
        gate = g.tensor("blk.0.ffn_gate_exps.weight")
        assert gate.dims == (64, 96, 4) and gate.type_id == MXFP4 and gate.nbytes == 64 * 96 * 4 // 32 * 17
        assert gate.bytes().tobytes() == banks["ffn_gate_exps"]
        assert g.tensor("blk.0.ffn_down_exps.weight").bytes().tobytes() == banks["ffn_down_exps"]
        r = g.tensor("blk.0.ffn_gate_inp.weight")
        assert r.dims == (64, 4) and r.type_id == F32 and r.bytes().tobytes() == banks["router"]
        assert g.tensor("blk.0.q4.weight").bytes().tobytes() == banks["q4"]
        assert not g.has("blk.1.ffn_gate_exps.weight")
        with pytest.raises(KeyError):
            g.tensor("blk.1.ffn_gate_exps.weight")


def test_every_expert_slice_is_where_an_independent_reader_finds_it(tmp_path):
    """tests/mapped_model.rs:36-118: each expert's bytes, found by an ordinary seek and read of
    the file (not through the mapping), equal the slice's; the slices tile the bank."""
    w, banks = model_writer(H=96, I=64, E=5)
    path = str(tmp_path / "m.gguf")
    w.write(path)
    with GgufFile(path) as g, open(path, "rb") as f:
        for name in ("ffn_gate_exps", "ffn_up_exps", "ffn_down_exps"):
            parent = g.tensor(f"blk.0.{name}.weight")
            per = parent.nbytes // 5
            ends = []
            for e in range(5):
                s = g.slice_last(parent.name, e)
                assert s.dims == parent.dims[:-1] and s.type_id == MXFP4 and s.nbytes == per
                assert s.offset == parent.offset + e * per
                f.seek(s.offset)
                assert f.read(s.nbytes) == s.bytes().tobytes() == banks[name][e * per:(e + 1) * per]
                ends.append(s.offset + s.nbytes)
            assert ends[-1] == parent.offset + parent.nbytes
        q = g.slice_last("blk.0.q4.weight", 1)
        assert q.dims == (32, 3) and q.nbytes == 3 * 18 and q.bytes().tobytes() == banks["q4"][54:108]


def test_slices_are_refused_where_they_do_not_exist(tmp_path):
    w = W.GgufWriter()
    w.add_tensor("vec", (64,), F32, bytes(256))
    w.add_tensor("half_blocks", (16, 1, 2), Q4_0, bytes(18))  # one block in all, half a block a slice
    w.add_tensor("bank", (32, 2, 3), Q4_0, bytes(6 * 18))
    path = str(tmp_path / "s.gguf")
    w.write(path)
    with GgufFile(path) as g:
        with pytest.raises(ValueError, match="no dimension"):
            g.slice_last("vec", 0)
        with pytest.raises(ValueError, match="not whole blocks"):
            g.slice_last("half_blocks", 0)
        with pytest.raises(ValueError):
            g.slice_last("bank", 3)
        with pytest.raises(ValueError):
            g.slice_last("absent", 0)
        assert g.slice_last("bank", 2).nbytes == 2 * 18


def test_general_alignment_moves_the_blob(tmp_path):
    w, banks = model_writer(alignment=256)
    path = str(tmp_path / "a.gguf")
    w.write(path)
    with GgufFile(path) as g:
        assert g.alignment == 256
        for t in g.tensors():
            assert t.offset % 256 == 0
        assert g.tensor("blk.0.ffn_up_exps.weight").bytes().tobytes() == banks["ffn_up_exps"]
    # version 2 reads the same way
    w.version = 2
    w.write(path)
    with GgufFile(path) as g:
        assert g.version == 2 and g.tensor("blk.0.q4.weight").bytes().tobytes() == banks["q4"]


def header(n_tensors, n_kv, version=3):
    return b"GGUF" + struct.pack("<IQQ", version, n_tensors, n_kv)


@pytest.mark.parametrize("case,raw,why", [
    ("magic", b"GGML" + bytes(60), "bad magic"),
    ("v1", header(0, 0, 1) + bytes(64), "version 1"),
    ("v4", header(0, 0, 4) + bytes(64), "version 4"),
    ("short", b"GGUF\x03\x00", "truncated"),
    ("kv_count", header(0, 1 << 50) + bytes(64), "implausible metadata key count"),
    ("tensor_count", header(1 << 50, 0) + bytes(64), "implausible tensor count"),
    ("nested", header(0, 1) + W.gstr("k") + struct.pack("<IIQ", W.ARRAY, W.ARRAY, 0) + bytes(32), "nested array"),
    ("vtype", header(0, 1) + W.gstr("k") + struct.pack("<I", 13) + bytes(32), "bad value type"),
    ("etype", header(0, 1) + W.gstr("k") + struct.pack("<IIQ", W.ARRAY, 77, 1) + bytes(32), "bad array element type"),
    ("array_len", header(0, 1) + W.gstr("k") + struct.pack("<IIQ", W.ARRAY, W.U32, 1 << 40) + bytes(32), "overruns"),
    ("string_len", header(0, 1) + struct.pack("<Q", 1 << 40) + bytes(64), "oversized key"),
    ("value_len", header(0, 1) + W.gstr("k") + struct.pack("<IQ", W.STRING, 1 << 20) + bytes(64), "string value"),
    ("rank0", header(1, 0) + W.tensor_info("t", (), F32, 0) + bytes(64), "rank 0"),
    ("rank5", header(1, 0) + W.tensor_info("t", (1, 1, 1, 1, 1), F32, 0) + bytes(64), "rank 5"),
    ("type", header(1, 0) + W.tensor_info("t", (32,), 5, 0) + bytes(256), "unknown type id 5"),
    ("blocks", header(1, 0) + W.tensor_info("t", (33,), MXFP4, 0) + bytes(256), "not whole blocks"),
    ("overrun", header(1, 0) + W.tensor_info("t", (64,), F32, 0) + bytes(40), "runs past the end"),
    ("offset", header(1, 0) + W.tensor_info("t", (4,), F32, 1 << 62) + bytes(64), "runs past the end"),
    ("align0", header(0, 1) + W.kv("general.alignment", W.U32, 0) + bytes(32), "power of two"),
    ("align3", header(0, 1) + W.kv("general.alignment", W.U32, 3) + bytes(32), "power of two"),
    ("align_neg", header(0, 1) + W.kv("general.alignment", W.I32, -32) + bytes(32), "positive integer"),
    ("align_str", header(0, 1) + W.kv("general.alignment", W.STRING, "32") + bytes(32), "positive integer"),
])
def test_malformed_files_are_refused(tmp_path, case, raw, why):
    path = str(tmp_path / f"{case}.gguf")
    with open(path, "wb") as f:
        f.write(raw)
    with pytest.raises(GgufError, match=why):
        GgufFile(path)


def test_a_truncated_file_is_refused_wherever_it_is_cut(tmp_path):
    """Cut a well-formed file at points in the header, the tensor index and the data blob:
    every cut is refused at open (the blob check catches what the header parse cannot)."""
    w, _ = model_writer()
    raw, data_off, offs = w.build()
    path = str(tmp_path / "t.gguf")
    for cut in (10, 30, 200, data_off - 20, data_off + 5, len(raw) - 1):
        with open(path, "wb") as f:
            f.write(raw[:cut])
        with pytest.raises(GgufError):
            GgufFile(path)
    with pytest.raises(GgufError, match="cannot open"):
        GgufFile(str(tmp_path / "absent.gguf"))


def test_a_repeated_key_keeps_the_later_value(tmp_path):
    w = W.GgufWriter()
    w.add("x", W.U32, 1).add("x", W.U32, 2)
    path = str(tmp_path / "r.gguf")
    w.write(path)
    with GgufFile(path) as g:
        assert g.u64("x") == 2 and g.n_tensors == 0


def test_the_mapping_outlives_a_rename_of_the_file(tmp_path):
    """The mapping holds the bytes: renaming the file after open does not disturb reads."""
    w, banks = model_writer()
    path = str(tmp_path / "m.gguf")
    w.write(path)
    g = GgufFile(path)
    os.rename(path, str(tmp_path / "moved.gguf"))
    assert g.tensor("blk.0.ffn_gate_exps.weight").bytes().tobytes() == banks["ffn_gate_exps"]
    g.close()


def test_moe_layout_sizes_the_expert_pool(tmp_path):
    """The expert half of the reference's ModelInfo (lib.rs:142-230): the blocks with stacked
    banks, one expert's bytes, and the expert / dense split of the weights."""
    H, I, E = 64, 96, 4
    w, banks = model_writer(H=H, I=I, E=E)
    w.add("gpt-oss.block_count", W.U32, 2)
    w.add_tensor("blk.1.ffn_gate_exps.weight", (H, I, E), MXFP4, bytes(H * I * E // 32 * 17))
    w.add_tensor("blk.1.ffn_up_exps.weight", (H, I, E), MXFP4, bytes(H * I * E // 32 * 17))
    w.add_tensor("blk.1.ffn_down_exps.weight", (I, H, E), MXFP4, bytes(H * I * E // 32 * 17))
    w.add_tensor("output_norm.weight", (H,), F32, bytes(4 * H))
    path = str(tmp_path / "m.gguf")
    w.write(path)
    with GgufFile(path) as g:
        lay = moe_layout(g)
        per = 3 * H * I // 32 * 17
        assert (lay.architecture, lay.block_count, lay.moe_blocks) == ("gpt-oss", 2, (0, 1))
        assert (lay.n_expert, lay.n_expert_used, lay.per_expert_bytes, lay.per_expert_uniform) == (E, 2, per, True)
        assert lay.expert_bytes == 2 * E * per
        assert lay.dense_bytes == 4 * H * E + 32 * 3 * 2 // 32 * 18 + 4 * H
    d = W.GgufWriter().add("general.architecture", W.STRING, "llama")
    d.write(str(tmp_path / "dense.gguf"))
    with GgufFile(str(tmp_path / "dense.gguf")) as g:
        with pytest.raises(ValueError, match="not a mixture of experts"):
            moe_layout(g)
