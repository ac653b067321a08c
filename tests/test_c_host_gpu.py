"""A host of the C ABI alone: beatlm_b200/c_host/vit_block.c, a C program
linked only against libbeatlm_b200.so (no Python, no PyTorch in its process,
no CUDA calls of its own), runs one ViT-S block (T=1370, D=384, 6 heads, MLP
1536, f16 weights by role, input U(-2, 2)) through plan -> arenas -> kernels
-> encode under the slice timer -> read back. Its output against the oracle's
block (crates/beatlm-bench/src/reference.rs:520-544) fed the weights as the
device holds them, within the f16 block bound of tests/test_block_gpu.py."""
import os
import subprocess

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

T, D, H, MLP = 1370, 384, 6, 1536
NAMES = ("norm1_g", "norm1_b", "qkv_w", "qkv_b", "proj_w", "proj_b", "ls1",
         "norm2_g", "norm2_b", "fc1_w", "fc1_b", "fc2_w", "fc2_b", "ls2")


def test_a_c_host_runs_a_vit_block_through_the_abi_alone(tmp_path):
    from beatlm_b200 import build
    from beatlm_b200.model import block_weights_by_role
    exe = build.build_c_host()
    w = block_weights_by_role(300, D, MLP, uniform=oracle.uniform)
    x = oracle.uniform(21, T * D, -2.0, 2.0)
    inp, out = tmp_path / "block.in", tmp_path / "block.out"
    with open(inp, "wb") as f:
        f.write(np.array([T, D, H, MLP], np.int32).tobytes())
        f.write(x.astype(np.float32).tobytes())
        for k in NAMES:
            f.write(np.asarray(w[k], np.float32).tobytes())
    env = {k: v for k, v in os.environ.items() if not k.startswith("PYTHON")}
    r = subprocess.run([exe, str(inp), str(out)], capture_output=True, text=True, env=env,
                       timeout=300)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    lines = r.stdout.splitlines()
    assert lines[-1] == "ok"
    assert [ln.split()[0] for ln in lines[1:8]] == ["norm1", "qkv", "attention", "proj", "norm2",
                                                   "fc1", "fc2"]
    got = np.fromfile(out, np.float32)
    rounded = dict(w)
    for k in ("qkv_w", "proj_w", "fc1_w", "fc2_w"):
        rounded[k] = oracle.round_f16(w[k])
    want = oracle.vit_block(x, rounded, T, H, 64, MLP, 1e-6, qkv_round="qk_f16")
    rel = float(np.linalg.norm(got.astype(np.float64) - want) / np.linalg.norm(want))
    print("C host block: rel-L2 %.3e" % rel)
    assert rel <= 1e-3
