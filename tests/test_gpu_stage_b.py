"""Stage B on the GPU: the streaming packer with the device kernels (uint32 word
packing, MXFP RTN) against the REAL reference packer's output, and the artifact
validator with device dequantization."""

import json

import pytest
import torch

from golden.make_stack_golden import packed_summary, write_checkpoint
from test_stream_pack_cpu import _artifacts_from_fixture

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("variant", ["packed", "packed_rtn"])
def test_stream_pack_on_device_matches_reference(variant, tmp_path, golden):
    from mlx_gptq_b200 import stream_pack

    fx = golden("stack_mxfp4")
    drop = json.loads(bytes(fx["packed_rtn_dropped"]).decode()) if variant == "packed_rtn" else []
    model_dir = write_checkpoint(str(tmp_path / "model"))
    calib = str(tmp_path / "calib")
    _artifacts_from_fixture(fx, calib, drop)
    mlx_dir = str(tmp_path / "mlx")
    packer = stream_pack.StreamingPacker(model_dir, calib, mlx_dir, "mxfp4", 4, 32, stream_pack.DEFAULT_EXCLUDE,
                                         device="cuda")
    packer.run()
    got, ref = packed_summary(mlx_dir), json.loads(bytes(fx[variant]).decode())
    assert sorted(got["tensors"]) == sorted(ref["tensors"])
    bad = [k for k in ref["tensors"] if got["tensors"][k] != ref["tensors"][k]]
    assert not bad, bad[:5]
    assert got["weight_map"] == ref["weight_map"] and got["quantization"] == ref["quantization"]


def test_validate_on_device(tmp_path, golden):
    """The reference's own Stage A artifacts respect the range guard against their source
    (verified); a scale byte past the exponent range is reported."""
    import safetensors.torch as st

    from mlx_gptq_b200 import validate

    fx = golden("stack_mxfp4")
    model_dir = write_checkpoint(str(tmp_path / "model"))
    calib = str(tmp_path / "calib")
    _artifacts_from_fixture(fx, calib)
    r = validate.validate(model_dir, calib, device="cuda")
    assert r["status"] == "verified" and not r["failures"] and r["tensors"] == 56
    assert all(w["ratio"] <= 1.0 for w in r["worst"])
    name = "model.layers.0.self_attn.q_proj.weight"
    blob = st.load_file(f"{calib}/layer_0000.safetensors")
    blob[f"{name}.scales"] = torch.full_like(blob[f"{name}.scales"], 254)
    st.save_file(blob, f"{calib}/layer_0000.safetensors")
    r = validate.validate(model_dir, calib, device="cuda")
    assert r["status"] == "failed" and [f["name"] for f in r["failures"]] == [name]
