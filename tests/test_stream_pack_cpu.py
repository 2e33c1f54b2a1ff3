"""Stage B streaming packer (mlx_gptq_b200.stream_pack) against the REAL reference's
output (mlx_gptq/stream_pack.py run by tests/golden/make_stack_golden.py on the
reference's own Stage A artifacts of a tiny Qwen3-MoE checkpoint).

The artifacts are rebuilt from the fixture's codes and scales, the packer runs on the
CPU with the oracle's numpy restatements of the two device kernels it calls (uint32
word packing, MXFP RTN), and every output tensor must match the reference bit for bit
(dtype, shape, sha256), as must the index's weight map and the config's quantization
entry; also with one stacked projection left to the RTN fallback."""

import json
import os

import numpy as np
import pytest
import torch

from golden.make_stack_golden import packed_summary, write_checkpoint


def _np_pack_q(q, bits):
    from oracle.packing import pack_q

    return torch.from_numpy(pack_q(q.cpu().numpy(), bits))


def _np_rtn_mxfp(w, mode):
    from oracle.grid import rtn_quantize_mxfp

    q, s, b, dq = rtn_quantize_mxfp(w.cpu().numpy(), mode)
    return torch.from_numpy(q), torch.from_numpy(s), None, torch.from_numpy(dq)


def _np_pack_nibbles(q):
    from oracle.packing import pack_nibbles

    return torch.from_numpy(pack_nibbles(q.cpu().numpy()))


def _np_unpack_nibbles(p):
    from oracle.packing import unpack_nibbles

    return torch.from_numpy(unpack_nibbles(p.cpu().numpy()))


def _artifacts_from_fixture(fx, out_dir, drop=()):
    from mlx_gptq_b200.artifacts import ArtifactWriter

    meta = json.loads(bytes(fx["meta"]).decode())
    w = ArtifactWriter(out_dir, {"mode": "mxfp4", "bits": 4, "group_size": 32, "storage_dtype": "bfloat16"})
    by_layer = {}
    for name, m in meta.items():
        if name in drop:
            continue
        li = int(name.split(".")[2])
        q = torch.from_numpy(fx[f"q:{name}"])
        s = torch.from_numpy(fx[f"s:{name}"])
        info = {"bits": 4, "group_size": 32, "mode": "mxfp4", "kind": m["kind"], "out_features": q.shape[0],
                "in_features": q.shape[1], "tokens": m["tokens"], "rel_err": m["rel_err"]}
        by_layer.setdefault(li, ({}, {}))
        by_layer[li][0][name] = (q, s, None)
        by_layer[li][1][name] = info
    for li in sorted(by_layer):
        w.write_layer(li, *by_layer[li])


@pytest.mark.parametrize("variant", ["packed", "packed_rtn"])
def test_stream_pack_matches_reference(variant, tmp_path, monkeypatch, golden):
    from mlx_gptq_b200 import artifacts, stream_pack

    monkeypatch.setattr(artifacts, "pack_nibbles", _np_pack_nibbles)
    monkeypatch.setattr(artifacts, "unpack_nibbles", _np_unpack_nibbles)
    monkeypatch.setattr(stream_pack, "pack_q", _np_pack_q)
    monkeypatch.setattr(stream_pack, "rtn_quantize_mxfp", _np_rtn_mxfp)
    fx = golden("stack_mxfp4")
    drop = json.loads(bytes(fx["packed_rtn_dropped"]).decode()) if variant == "packed_rtn" else []
    model_dir = write_checkpoint(str(tmp_path / "model"))
    calib = str(tmp_path / "calib")
    _artifacts_from_fixture(fx, calib, drop)
    mlx_dir = str(tmp_path / "mlx")
    packer = stream_pack.StreamingPacker(model_dir, calib, mlx_dir, "mxfp4", 4, 32, stream_pack.DEFAULT_EXCLUDE,
                                         device="cpu")
    packer.run()
    got, ref = packed_summary(mlx_dir), json.loads(bytes(fx[variant]).decode())
    assert sorted(got["tensors"]) == sorted(ref["tensors"])
    bad = [k for k in ref["tensors"] if got["tensors"][k] != ref["tensors"][k]]
    assert not bad, bad[:5]
    assert got["weight_map"] == ref["weight_map"] and got["quantization"] == ref["quantization"]
    assert packer.stats["rtn"] == (1 if drop else 0)


def test_stream_pack_rejects_unused_artifacts_and_mismatched_bits(tmp_path, monkeypatch, golden):
    from mlx_gptq_b200 import artifacts, stream_pack

    monkeypatch.setattr(artifacts, "pack_nibbles", _np_pack_nibbles)
    monkeypatch.setattr(artifacts, "unpack_nibbles", _np_unpack_nibbles)
    monkeypatch.setattr(stream_pack, "pack_q", _np_pack_q)
    monkeypatch.setattr(stream_pack, "rtn_quantize_mxfp", _np_rtn_mxfp)
    fx = golden("stack_mxfp4")
    model_dir = write_checkpoint(str(tmp_path / "model"))
    calib = str(tmp_path / "calib")
    # one expert's down_proj missing: layer 1's other down_proj artifacts go unused
    drop = ["model.layers.1.mlp.experts.3.down_proj.weight"]
    _artifacts_from_fixture(fx, calib, drop)
    with pytest.raises(RuntimeError, match="not consumed"):
        stream_pack.StreamingPacker(model_dir, calib, str(tmp_path / "mlx"), "mxfp4", 4, 32,
                                    stream_pack.DEFAULT_EXCLUDE, device="cpu").run()
    with pytest.raises(RuntimeError, match="!= config"):
        stream_pack.StreamingPacker(model_dir, calib, str(tmp_path / "mlx8"), "mxfp8", 8, 32,
                                    stream_pack.DEFAULT_EXCLUDE, device="cpu").run()
    assert stream_pack.sanitize_name("model.language_model.layers.0.x", True) == "model.layers.0.x"
    assert stream_pack.sanitize_name("model.visual.blocks.0.w", False) is None
    assert stream_pack.unit_of("model.layers.12.mlp.gate.weight") == "layer.0012"
