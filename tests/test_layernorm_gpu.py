"""The standalone LayerNorm (reference.rs:247-270; WGSL layer_norm
wgsl.rs:519-585) through the C ABI against the oracle: the 16-byte-access
form (column counts and strides that are multiples of 4) and the scalar form
(the others), f32 and 16-bit outputs, row grouping (the final norm's
TokensToMap), and row parts equal to the whole.

Tolerance: the reference's per-element |d| <= 1e-4 + 1e-4 |ref| for f32
outputs (reference.rs:17-24); 16-bit outputs within one unit of the
output type's last place of the oracle's value."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


def _run(rows, cols, out_dtype="f32", ldx=None, seed=0, rows_part=None):
    import torch
    from beatlm_b200 import ops
    rng = np.random.default_rng(seed)
    ldx = ldx or cols
    x = (rng.standard_normal((rows, ldx), dtype=np.float32) * 3 + 0.5).astype(np.float32)
    g = rng.uniform(0.8, 1.2, cols).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, cols).astype(np.float32)
    td = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[out_dtype]
    xd = torch.from_numpy(x).cuda()[:, :cols]
    out = torch.zeros((rows, cols), dtype=td, device="cuda")
    ops.layernorm(xd, torch.from_numpy(g).cuda(), torch.from_numpy(b).cuda(), 1e-6, out=out)
    want = oracle.layernorm(np.ascontiguousarray(x[:, :cols]).ravel(), g, b, 1e-6)
    return out.float().cpu().numpy(), want.reshape(rows, cols)


@pytest.mark.parametrize("cols", [384, 1024, 128, 640])
@pytest.mark.parametrize("rows", [1, 5, 1370])
def test_vector_form_matches_the_oracle(rows, cols):
    got, want = _run(rows, cols, seed=rows + cols)
    assert np.all(np.abs(got - want) <= 1e-4 + 1e-4 * np.abs(want))


@pytest.mark.parametrize("cols,ldx", [(383, 383), (100, 130), (1022, 1024)])
def test_scalar_form_matches_the_oracle(cols, ldx):
    got, want = _run(257, cols, ldx=ldx, seed=cols)
    assert np.all(np.abs(got - want) <= 1e-4 + 1e-4 * np.abs(want))


@pytest.mark.parametrize("out_dtype,ulp", [("f16", 2.0 ** -10), ("bf16", 2.0 ** -7)])
@pytest.mark.parametrize("cols", [384, 1024, 383])
def test_16bit_outputs(out_dtype, ulp, cols):
    got, want = _run(300, cols, out_dtype=out_dtype, seed=3)
    assert np.all(np.abs(got - want) <= ulp * np.maximum(np.abs(want), 2.0 ** -14) + 1e-6)


def test_row_groups_and_parts_equal_the_whole():
    """The final norm reads patch rows only (TokensToMap, kernel.rs:703-720):
    rows grouped T-1 at a time after one class row. Split into row parts
    (Program::split), the parts give the whole result bit for bit."""
    import torch
    from beatlm_b200 import ops
    from beatlm_b200.runtime import Kernels, Spec
    frames, t, d = 2, 1370, 384
    rng = np.random.default_rng(8)
    x = rng.standard_normal((frames * t, d), dtype=np.float32)
    g, b = np.ones(d, np.float32), np.zeros(d, np.float32)
    xd, gd, bd = (torch.from_numpy(a).cuda() for a in (x, g, b))
    out = torch.zeros((frames * (t - 1), d), dtype=torch.float32, device="cuda")
    ops.layernorm(xd, gd, bd, 1e-6, out=out, in_row_offset=1, in_group=(t - 1, 1))
    want = np.concatenate([oracle.layernorm(x[f * t + 1:(f + 1) * t].ravel(), g, b, 1e-6)
                           .reshape(t - 1, d) for f in range(frames)])
    got = out.cpu().numpy()
    assert np.all(np.abs(got - want) <= 1e-4 + 1e-4 * np.abs(want))
    parts = torch.zeros_like(out)
    k = Kernels([Spec(ops.layernorm_args(xd, gd, bd, 1e-6, out=parts, in_row_offset=1,
                                         in_group=(t - 1, 1)), "norm", 7)])
    k.encode_all()
    torch.cuda.synchronize()
    assert torch.equal(parts, out)
