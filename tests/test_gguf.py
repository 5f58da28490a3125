"""GGUF checkpoint reader (dcpp_gguf_*) and model binding from GGUF, on CPU.

Files are written with gguf-py 0.19.0 (the library the reference's converter,
utils/convert-model/src/convert_hf_safetensors_to_gguf.py, writes them with)
and read back through the C ABI; gguf-py's GGUFReader is the check for the
parse (tensor names, types, dimensions, data offsets, bytes, metadata).
Binding is checked through host-only Flux2 models (dcpp_flux2_create_host):
load_gguf must assemble exactly what set_param assembles from the same bytes,
tensor-parallel shards included.  The reference's behaviour kept: tensors the
model does not know are skipped (GGUFLoaderVisitor::validate only reports
them), a parameter absent from the file fails with "Tensor not found", a
shape mismatch names the tensor.
"""

import gguf
import numpy as np
import pytest
from gguf import GGMLQuantizationType as Q

import dcpp_b200
import flux2_oracle as fo
import tp_oracle as tpo
from dcpp_b200 import synth
from gguf_util import _raw, write_gguf

NOT_FOUND, INVALID, UNSUPPORTED = 8, 1, 2


def flux_cfg(heads=4, **kw):
    base = dict(num_layers=1, num_single_layers=1, num_attention_heads=heads, attention_head_dim=128,
                joint_attention_dim=64, in_channels=32, timestep_guidance_channels=256, guidance_embeds=True)
    base.update(kw)
    return synth.Flux2Cfg(**base)


KV = {
    "general.name": ("string", "flux2-test"),
    "test.u32": ("uint32", 4000000000),
    "test.i32": ("int32", -7),
    "test.u8": ("uint8", 200),
    "test.i16": ("int16", -300),
    "test.u64": ("uint64", 1 << 40),
    "test.i64": ("int64", -(1 << 40)),
    "test.f32": ("float32", 1.5),
    "test.f64": ("float64", -2.25),
    "test.bool": ("bool", True),
    "test.ints": ("array", [1, -2, 3]),
    "test.floats": ("array", [0.5, 1.25]),
    "test.strs": ("array", ["a", "", "longer string é"]),
}


@pytest.mark.parametrize("alignment", [None, 64, 256])
def test_reader_matches_gguf_py(tmp_path, alignment):
    rng = np.random.default_rng(3)
    params = {
        "v.f32": (fo.GGML_F32, (5,), rng.standard_normal(5).astype(np.float32).tobytes()),
        "m.f16": (fo.GGML_F16, (3, 8), rng.standard_normal(24).astype(np.float16).tobytes()),
        "m.bf16": (fo.GGML_BF16, (2, 16), rng.integers(0, 256, 64, dtype=np.uint8).tobytes()),
        "m.q8": (fo.GGML_Q8_0, (4, 64), rng.integers(0, 256, 4 * 2 * 34, dtype=np.uint8).tobytes()),
        "m.q4k": (fo.GGML_Q4_K, (3, 512), rng.integers(0, 256, 3 * 2 * 144, dtype=np.uint8).tobytes()),
        "t.3d": (fo.GGML_F32, (2, 3, 4), rng.standard_normal(24).astype(np.float32).tobytes()),
        "t.unit": (fo.GGML_F32, (1,), np.float32([7]).tobytes()),
    }
    path = write_gguf(tmp_path / "a.gguf", params, alignment=alignment, kv=KV)
    ref = gguf.GGUFReader(path)
    with dcpp_b200.GGUFFile(path) as f:
        info = f.info()
        assert info["version"] == 3
        assert info["alignment"] == ref.alignment
        assert info["data_offset"] == ref.data_offset
        ts = f.tensors()
        assert [t["name"] for t in ts] == [t.name for t in ref.tensors]
        for mine, theirs in zip(ts, ref.tensors):
            assert mine["type"] == int(theirs.tensor_type)
            assert mine["ne"] == tuple(int(x) for x in theirs.shape)
            assert mine["offset"] == theirs.data_offset
            assert mine["offset"] % ref.alignment == 0
            assert mine["nbytes"] == theirs.n_bytes
            got = f.tensor_bytes(mine["name"])
            assert got.tobytes() == np.asarray(theirs.data).tobytes()
            assert got.tobytes() == _raw(params[mine["name"]][2])
        meta = f.metadata()
        want = {k: fld.contents() for k, fld in ref.fields.items() if not k.startswith("GGUF.")}
        assert set(meta) == set(want)
        for k, (kind, v) in meta.items():
            if isinstance(v, float) or (isinstance(v, list) and v and isinstance(v[0], float)):
                assert np.allclose(v, want[k]), k
            else:
                assert v == want[k], (k, v, want[k])
        assert meta["test.strs"][0] == "array[string]"
        assert meta["test.u8"][0] == "u8" and meta["test.bool"] == ("bool", True)
        assert f.find("m.q8") == 3 and f.find("nope") == -1


def test_type_sizes_match_ggml_traits(tmp_path):
    """Every type the reader sizes: its byte count equals gguf-py's for a row of
    two blocks (the table is ggml's type traits)."""
    rng = np.random.default_rng(0)
    types = [Q.F32, Q.F16, Q.Q4_0, Q.Q4_1, Q.Q5_0, Q.Q5_1, Q.Q8_0, Q.Q8_1, Q.Q2_K, Q.Q3_K, Q.Q4_K, Q.Q5_K,
             Q.Q6_K, Q.Q8_K, Q.I8, Q.I16, Q.I32, Q.I64, Q.F64, Q.BF16]
    params = {}
    for t in types:
        blk, nb = gguf.GGML_QUANT_SIZES[t]
        params[f"t{int(t)}"] = (int(t), (3, 2 * blk), rng.integers(0, 256, 3 * 2 * nb, dtype=np.uint8).tobytes())
    w = gguf.GGUFWriter(str(tmp_path / "types.gguf"), arch="x")
    for name, (gt, shape, data) in params.items():
        w.add_tensor(name, np.frombuffer(data, np.uint8).reshape(3, -1), raw_dtype=Q(gt))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    ref = {t.name: t for t in gguf.GGUFReader(str(tmp_path / "types.gguf")).tensors}
    with dcpp_b200.GGUFFile(tmp_path / "types.gguf") as f:
        for t in f.tensors():
            assert t["nbytes"] == ref[t["name"]].n_bytes, t["name"]
            assert f.tensor_bytes(t["name"]).tobytes() == params[t["name"]][2]


def _flux_names(c, full, rank, n):
    return list(tpo.expected_shards(c, full, rank, n)) + list(tpo.vector_names(c))


# (heads, tp size, weight type, split GGUF names)
LOADS = [(4, 1, fo.GGML_Q8_0, False), (4, 1, fo.GGML_Q4_K, True), (6, 2, fo.GGML_Q4_K, False),
         (4, 2, fo.GGML_Q8_0, True)]


@pytest.mark.parametrize("heads,n,wtype,split", LOADS)
def test_load_gguf_equals_set_param(tmp_path, heads, n, wtype, split):
    c = flux_cfg(heads)
    params = synth.make_params(c, wtype, seed=11, split=split)
    path = write_gguf(tmp_path / "transformer.gguf", params)
    full = fo.Weights(params)
    for rank in range(n):
        a = dcpp_b200.Flux2Model(None, c, tp_rank=rank, tp_size=n)
        a.load_params(params)
        b = dcpp_b200.Flux2Model(None, c, tp_rank=rank, tp_size=n)
        bound, unused = b.load_gguf(path)
        assert (bound, unused) == (len(params), 0)
        assert b.missing() == (0, "")
        for name in _flux_names(c, full, rank, n):
            ta, sa, ba = a.read_param(name)
            tb, sb, bb = b.read_param(name)
            assert (ta, sa) == (tb, sb), name
            assert ba.tobytes() == bb.tobytes(), name
        a.close()
        b.close()


def test_load_gguf_skips_unknown_and_reports_missing(tmp_path):
    c = flux_cfg()
    params = synth.make_params(c, fo.GGML_Q8_0, seed=2)
    extra = dict(params)
    extra["some.unused.tensor"] = (fo.GGML_F32, (4,), np.zeros(4, np.float32).tobytes())
    m = dcpp_b200.Flux2Model(None, c)
    assert m.load_gguf(write_gguf(tmp_path / "extra.gguf", extra)) == (len(params), 1)
    m.close()

    dropped = sorted(params)[3]
    less = {k: v for k, v in params.items() if k != dropped}
    m = dcpp_b200.Flux2Model(None, c)
    with pytest.raises(dcpp_b200.DcppError) as e:
        m.load_gguf(write_gguf(tmp_path / "less.gguf", less))
    assert e.value.status == NOT_FOUND
    assert "Tensor not found" in str(e.value)
    m.close()


def test_load_gguf_shape_mismatch_names_tensor(tmp_path):
    c = flux_cfg()
    params = synth.make_params(c, fo.GGML_Q8_0, seed=4)
    bad = dict(params)
    gt, shape, data = params["proj_out.weight"]
    # Same bytes, rows and columns swapped in the header.
    assert len(shape) == 2
    raw = np.frombuffer(_raw(data), np.uint8)
    if gt == fo.GGML_BF16:
        bad["proj_out.weight"] = (gt, (shape[1], shape[0]), raw.tobytes())
    else:
        bad["proj_out.weight"] = (fo.GGML_F32, (shape[0] * shape[1] // 64, 64),
                                  np.zeros(shape[0] * shape[1], np.float32)[: shape[0] * shape[1] // 64 * 64].tobytes())
    m = dcpp_b200.Flux2Model(None, c)
    with pytest.raises(dcpp_b200.DcppError) as e:
        m.load_gguf(write_gguf(tmp_path / "bad.gguf", bad))
    assert "proj_out" in str(e.value)
    m.close()


def test_directory_resolution(tmp_path):
    p = {"x": (fo.GGML_F32, (2,), np.float32([1, 2]).tobytes())}
    q = {"y": (fo.GGML_F32, (2,), np.float32([3, 4]).tobytes())}
    d = tmp_path / "component"
    d.mkdir()
    write_gguf(d / "b.gguf", q)
    write_gguf(d / "a.gguf", p)
    (d / "config.json").write_text("{}")
    with dcpp_b200.GGUFFile(d) as f:  # first *.gguf in name order
        assert [t["name"] for t in f.tensors()] == ["x"]
    empty = tmp_path / "empty"
    empty.mkdir()
    for missing in (empty, tmp_path / "nope"):
        with pytest.raises(dcpp_b200.DcppError) as e:
            dcpp_b200.GGUFFile(missing)
        assert e.value.status == NOT_FOUND and "No such GGUF file in path" in str(e.value)


def _expect_invalid(path, fragment):
    with pytest.raises(dcpp_b200.DcppError) as e:
        dcpp_b200.GGUFFile(path)
    assert e.value.status in (INVALID, UNSUPPORTED), e.value
    assert fragment in str(e.value), str(e.value)


def test_corrupt_files_fail_cleanly(tmp_path):
    rng = np.random.default_rng(9)
    params = {"m.q8": (fo.GGML_Q8_0, (4, 64), rng.integers(0, 256, 4 * 2 * 34, dtype=np.uint8).tobytes()),
              "v": (fo.GGML_F32, (8,), np.ones(8, np.float32).tobytes())}
    good = open(write_gguf(tmp_path / "good.gguf", params, kv=KV), "rb").read()
    ref = gguf.GGUFReader(str(tmp_path / "good.gguf"))
    bad = tmp_path / "bad.gguf"

    bad.write_bytes(b"GGUX" + good[4:])
    _expect_invalid(bad, "bad magic")
    bad.write_bytes(good[:4] + (1).to_bytes(4, "little") + good[8:])
    _expect_invalid(bad, "version 1")
    bad.write_bytes(good[:4] + (3 << 24).to_bytes(4, "little") + good[8:])
    _expect_invalid(bad, "big-endian")
    # Every cut inside the header and tensor infos: a clean "truncated" error.
    for cut in list(range(0, 64)) + list(range(64, ref.data_offset, 7)):
        bad.write_bytes(good[:cut])
        with pytest.raises(dcpp_b200.DcppError) as e:
            dcpp_b200.GGUFFile(bad)
        assert e.value.status == INVALID, (cut, str(e.value))
    # A cut inside the data section: the tensor is outside the file.
    bad.write_bytes(good[:-8])
    _expect_invalid(bad, "not within the file bounds")
    # A tensor count far beyond the file.
    bad.write_bytes(good[:8] + (1 << 60).to_bytes(8, "little") + good[16:])
    _expect_invalid(bad, "truncated")


def test_config_and_gguf_folder_layout(tmp_path):
    """from_pretrained's folder layout on the host: config.json parsed by
    dcpp_flux2_config_from_file, the GGUF found in the same folder."""
    c = flux_cfg(guidance_embeds=False)
    params = synth.make_params(c, fo.GGML_Q8_0, seed=8)
    d = tmp_path / "transformer"
    d.mkdir()
    write_gguf(d / "model.gguf", params)
    m = dcpp_b200.Flux2Model(None, c)
    assert m.load_gguf(d)[0] == len(params)
    assert m.missing() == (0, "")
    m.close()
