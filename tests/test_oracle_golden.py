"""Pin the CPU oracle to outputs of the reference's own kernel (tests/golden)."""
import os

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import rope_attn_oracle as O

K = np.load(os.path.join(GOLDEN, "golden_kernel.npz"))
CASES = sorted({k.split("/")[0] for k in K.files})


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_kernel(name):
    q, k, v = (K[f"{name}/{t}"] for t in "qkv")
    cos, sin, cu, ref = K[f"{name}/cos"], K[f"{name}/sin"], K[f"{name}/cu_seqlens"], K[f"{name}/out"]
    rd = None if q.dtype == np.float32 else str(q.dtype)
    # The reference kernel rounds rotated Q/K and P to the input type (fused_attn.py:344-345, 413).
    qr = O.apply_rope(q.astype(np.float32), cos, sin, rd)
    kr = O.apply_rope(k.astype(np.float32), cos, sin, rd)
    out = O.varlen_attention(qr, kr, v.astype(np.float32), cu, p_round=rd)
    err = np.abs(out - ref.astype(np.float32))
    tol = 2e-5 if rd is None else 2e-3
    assert err.max() < tol, (name, err.max())
    # the plain unfused fp32 oracle (no intermediate rounding) is within the bf16 budget
    out32 = O.rope_attention(q.astype(np.float32), k.astype(np.float32), v.astype(np.float32), cos, sin, cu)
    e32 = np.abs(out32 - ref.astype(np.float32))
    assert e32.max() < 2e-2 and e32.mean() < 2e-3, (name, e32.max(), e32.mean())


def test_round_to_bf16_is_rne():
    x = np.array([1.0, 1.00390625, 1.01171875, -3.0e-3, 65504.0, np.inf], dtype=np.float32)
    r = O.round_to(x, "bfloat16")
    import torch
    t = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(r, t)


def test_flops_bytes():
    cu = [0, 64, 128]
    assert O.attention_flops(cu, 16, 80) == 4 * 2 * 64 * 64 * 16 * 80
    assert O.attention_bytes(128, 2, 16, 80) == 4 * 128 * 16 * 80 * 2 + 2 * 128 * 40 * 4 + 12
