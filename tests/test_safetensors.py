"""Checkpoint reading for quantize-on-load (tensai_b200/safetensors.py, the
reference's encoding/safetensors package): files written by the Hugging Face
`safetensors` library read back bit for bit in every dtype the reference
reads, the header checks of safetensors.go:66-118, Save read back by the
library, and sharded checkpoints through an index. The GPU case quantizes a
BF16 Linear weight straight from the file and compares the codes and scales
with the oracle's QuantizeMatrix4 of the widened transpose."""
import json
import os
import struct

import numpy as np
import pytest

from tensai_b200 import safetensors as ST

st_numpy = pytest.importorskip("safetensors.numpy")


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_reads_library_files_in_every_dtype(tmp_path):
    rng = np.random.default_rng(1)
    t = {"a.f32": rng.standard_normal((3, 5)).astype(np.float32),
         "b.f16": rng.standard_normal((4, 2)).astype(np.float16),
         "c.f64": rng.standard_normal((7,)),
         "d.scalar": np.array(2.5, np.float32)}
    p = str(tmp_path / "x.safetensors")
    st_numpy.save_file(t, p, metadata={"format": "pt", "k": "v"})
    with ST.Open(p) as f:
        assert f.Names() == sorted(t)
        assert f.Metadata() == {"format": "pt", "k": "v"}
        assert f.Info("b.f16") == ("F16", [4, 2], True)
        assert f.Info("nope") == ("", None, False)
        assert np.array_equal(_bits(f.Tensor("a.f32")), _bits(t["a.f32"]))
        assert np.array_equal(_bits(f.Tensor("b.f16")), _bits(t["b.f16"].astype(np.float32)))
        assert np.array_equal(_bits(f.Tensor("c.f64")), _bits(t["c.f64"].astype(np.float32)))
        assert f.Tensor("d.scalar").shape == (1,) and f.Tensor("d.scalar")[0] == 2.5
        with pytest.raises(KeyError):
            f.Tensor("nope")


def test_bf16_widening(tmp_path):
    torch = pytest.importorskip("torch")
    from safetensors.torch import save_file
    w = torch.randn(6, 10, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
    p = str(tmp_path / "w.safetensors")
    save_file({"w": w}, p)
    with ST.Open(p) as f:
        assert f.Info("w")[0] == "BF16"
        assert np.array_equal(_bits(f.Tensor("w")), _bits(w.float().numpy()))


def test_f16_special_values(tmp_path):
    h = np.array([0.0, -0.0, 6e-8, -6e-8, 1e-5, 65504.0, np.inf, -np.inf, np.nan, 1.0, -2.5], np.float16)
    h = np.concatenate([h, np.arange(0, 1024, dtype=np.uint16).view(np.float16)])  # every subnormal
    p = str(tmp_path / "h.safetensors")
    st_numpy.save_file({"h": h}, p)
    with ST.Open(p) as f:
        assert np.array_equal(_bits(f.Tensor("h")), _bits(h.astype(np.float32)))


def _raw(header: bytes, data: bytes = b"") -> bytes:
    return struct.pack("<Q", len(header)) + header + data


@pytest.mark.parametrize("blob, msg", [
    (struct.pack("<Q", 0), "implausible header length"),
    (struct.pack("<Q", 200 << 20) + b"{}", "implausible header length"),
    (_raw(b"{not json"), "parsing header"),
    (_raw(json.dumps({"t": {"dtype": "F32", "shape": [2], "data_offsets": [8, 0]}}).encode()), "invalid offsets"),
    (_raw(json.dumps({"t": {"dtype": "F32", "shape": [-1], "data_offsets": [0, 0]}}).encode()), "negative dimension"),
    (_raw(json.dumps({"t": {"dtype": "F32", "shape": [3], "data_offsets": [0, 8]}}).encode(), b"\0" * 8),
     "does not match"),
])
def test_header_checks(tmp_path, blob, msg):
    p = tmp_path / "bad.safetensors"
    p.write_bytes(blob)
    with pytest.raises(ValueError, match=msg):
        ST.Open(str(p))


def test_unknown_dtype_is_listed_but_not_read(tmp_path):
    p = tmp_path / "i.safetensors"
    p.write_bytes(_raw(json.dumps({"t": {"dtype": "I32", "shape": [2], "data_offsets": [0, 8]}}).encode(), b"\0" * 8))
    with ST.Open(str(p)) as f:
        assert f.Info("t") == ("I32", [2], True)
        with pytest.raises(ValueError, match="unsupported dtype"):
            f.Tensor("t")


def test_save_reads_back_with_the_library(tmp_path):
    rng = np.random.default_rng(3)
    t = {"z": rng.standard_normal((2, 3)).astype(np.float32), "a": np.arange(5, dtype=np.float32)}
    p = str(tmp_path / "s.safetensors")
    ST.SaveFile(p, t, {"who": "tensai"})
    n = struct.unpack("<Q", open(p, "rb").read(8))[0]
    assert (8 + n) % 8 == 0  # the buffer starts 8-byte aligned
    back = st_numpy.load_file(p)
    assert set(back) == set(t) and all(np.array_equal(back[k], t[k]) for k in t)
    with ST.Open(p) as f:
        assert f.Metadata() == {"who": "tensai"} and f.Names() == ["a", "z"]
    with pytest.raises(ValueError, match="reserved"):
        ST.SaveFile(p, {"__metadata__": np.zeros(1, np.float32)})


def test_sharded_checkpoint(tmp_path):
    rng = np.random.default_rng(4)
    s1 = {"l0.w": rng.standard_normal((4, 4)).astype(np.float32)}
    s2 = {"l1.w": rng.standard_normal((2, 8)).astype(np.float32), "l1.b": np.ones(8, np.float32)}
    st_numpy.save_file(s1, str(tmp_path / "m-1.safetensors"))
    st_numpy.save_file(s2, str(tmp_path / "m-2.safetensors"))
    wm = {"l0.w": "m-1.safetensors", "l1.w": "m-2.safetensors", "l1.b": "m-2.safetensors"}
    idx = tmp_path / "model.safetensors.index.json"
    idx.write_text(json.dumps({"metadata": {}, "weight_map": wm}))
    with ST.OpenSharded(str(idx)) as s:
        assert s.Names() == sorted(wm)
        assert s.Info("l1.w") == ("F32", [2, 8], True)
        assert np.array_equal(s.Tensor("l0.w"), s1["l0.w"])
        assert np.array_equal(s.Tensor("l1.b"), s2["l1.b"])
    idx.write_text(json.dumps({"weight_map": {"l0.w": "m-2.safetensors"}}))
    with pytest.raises(ValueError, match="lacks it"):
        ST.OpenSharded(str(idx))
    idx.write_text(json.dumps({"weight_map": {}}))
    with pytest.raises(ValueError, match="no weight_map"):
        ST.OpenSharded(str(idx))


@pytest.mark.gpu
@pytest.mark.parametrize("bits", [4, 8])
def test_quantize_linear_from_bf16_file(tmp_path, bits):
    import torch
    from safetensors.torch import save_file

    from oracle import oracle as O
    from tensai_b200 import _lib
    from tensai_b200 import quant as Q
    torch.cuda.init()
    _lib.check(_lib.load().tq_set_device(0))
    out_f, in_f = 384, 200
    w = torch.from_numpy(O.synth((out_f, in_f), 71, 3, 0.05)).to(torch.bfloat16)
    p = str(tmp_path / "lin.safetensors")
    save_file({"model.layers.0.mlp.up_proj.weight": w}, p)
    with ST.Open(p) as f:
        h = f.QuantizeLinear("model.layers.0.mlp.up_proj.weight", bits)
    q, s = Q.download(h, bits, in_f, out_f)
    qo, so = (O.quantize8 if bits == 8 else O.quantize4)(np.ascontiguousarray(w.float().numpy().T))
    assert np.array_equal(q, qo) and np.array_equal(_bits(s), _bits(so))
    Q.free(h)
    assert os.path.exists(p)
