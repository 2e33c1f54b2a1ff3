"""Our Stage A command line against the REAL reference's layer-sequential run.

tests/golden/stack_mxfp4.npz holds the artifacts mlx_gptq.sequential.Pipeline wrote
on CPU (torch float32 solver) for a tiny seeded Qwen3-MoE checkpoint and token
windows (tests/golden/make_stack_golden.py). The same checkpoint is regenerated
here and calibrated on the GPU.

Layer 0 sees the reference's inputs (up to the bf16 rounding of an RMSNorm computed
on another device), so it is held to the north-star bar: >= 99.9% of codes identical
and every tensor's rel_err within 0.5% of the reference's. Layer 1's inputs come out
of our GPU forward of the quantized layer 0 instead of the reference's CPU forward:
the bf16 activations differ in the last bit for many rows and, where top-k routing
ties break differently, a few tokens reach another expert. Its bound is therefore the
measured drift, with margin: >= 95% of layer 1's codes and >= 97% over both layers,
E8M0 scales >= 97% over both layers, rel_err within 3%, and routed token counts within
1% in total. Measured on a B200: layer 0 99.908% of codes, worst rel_err deviation
0.12%; layer 1 96.52%, 0.55%; both layers 98.22%, scales 99.68%; 42 of 48 expert
token counts identical (6 of 6,144 routed rows moved).
"""

import json
import os

import numpy as np
import pytest

from golden.make_stack_golden import BATCH, write_checkpoint, windows

pytestmark = pytest.mark.gpu


def test_cli_matches_reference_stack(tmp_path, golden):
    from mlx_gptq_b200 import calibrate
    from mlx_gptq_b200.artifacts import ArtifactReader

    ref = golden("stack_mxfp4")
    meta = json.loads(bytes(ref["meta"]).decode())
    model_dir = write_checkpoint(str(tmp_path / "model"))
    toks = tmp_path / "t.npy"
    np.save(toks, windows())
    out = str(tmp_path / "out")
    calibrate.main(["--model", model_dir, "--output", out, "--calibration-tokens", str(toks), "--mode", "mxfp4",
                    "--devices", "cuda:0", "--batch-size", str(BATCH)])
    reader = ArtifactReader(out)
    assert sorted(reader.tensors) == sorted(meta)
    agree = {0: [0, 0], 1: [0, 0]}
    worst = {0: 0.0, 1: 0.0}
    s_agree = [0, 0]
    tok_same, n_exp, tok_diff, tok_total = 0, 0, 0, 0
    for name, m in meta.items():
        q, s, _, info = reader.get(name)
        rq, rs = ref[f"q:{name}"], ref[f"s:{name}"]
        layer = int(name.split(".")[2])
        agree[layer][0] += int((q.numpy() == rq).sum())
        agree[layer][1] += rq.size
        s_agree[0] += int((s.numpy() == rs).sum())
        s_agree[1] += rs.size
        worst[layer] = max(worst[layer], abs(info["rel_err"] - m["rel_err"]) / m["rel_err"])
        if m["kind"] == "expert":
            n_exp += 1
            tok_same += int(info["tokens"] == m["tokens"])
            tok_diff += abs(info["tokens"] - m["tokens"])
            tok_total += m["tokens"]
    a0, a1 = (agree[k][0] / agree[k][1] for k in (0, 1))
    a_all = (agree[0][0] + agree[1][0]) / (agree[0][1] + agree[1][1])
    print(f"codes agree: layer 0 {a0:.5f}, layer 1 {a1:.5f}, all {a_all:.5f}; scales {s_agree[0] / s_agree[1]:.5f}; "
          f"worst rel_err deviation: layer 0 {worst[0]:.4f}, layer 1 {worst[1]:.4f}; expert token counts equal "
          f"{tok_same}/{n_exp}, total deviation {tok_diff}/{tok_total}")
    assert a0 >= 0.999 and worst[0] <= 0.005  # identical inputs
    assert a_all >= 0.97 and a1 >= 0.95 and worst[1] <= 0.03  # inputs from our own forward
    assert s_agree[0] / s_agree[1] >= 0.97
    assert tok_diff <= 0.01 * tok_total, (tok_diff, tok_total)
