"""Generate the golden vectors in this folder from the reference itself.

Run in a container where the reference checkout is available:

    REFERENCE_DIR=/path/to/fused-rope-attn python tests/golden/make_golden.py

* host functions (compute_rope_2d, get_window_index, window_shuffle,
  window_unshuffle) run natively on CPU;
* the reference Triton kernel ``fused_attn_kernel`` runs on CPU under the Triton
  interpreter (``TRITON_INTERPRET=1``) by calling the JIT function behind the
  autotuner with an explicit BLOCK_M/BLOCK_N, since the wrapper refuses CPU
  tensors (fused_attn.py:159-160). The interpreter mis-handles bf16, so kernel
  goldens use fp16 and fp32 inputs.

Outputs: golden_host.npz and golden_kernel.npz (inputs + reference outputs).
Nothing at test time reads the reference; the tests only read these files.
"""
from __future__ import annotations

import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

REF = os.environ.get("REFERENCE_DIR", "/root/reference")
sys.path.insert(0, REF)
import fused_attn as R  # noqa: E402
import utils as RU  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))

HOST_GRIDS = {
    "g32x32": [(1, 32, 32)],
    "g22x30": [(1, 22, 30)],
    "g2x16x24": [(2, 16, 24)],
    "gmulti": [(1, 16, 16), (1, 8, 12), (3, 4, 6)],
    "g18x10": [(1, 18, 10)],
}


def host_goldens():
    out = {}
    for name, grid in HOST_GRIDS.items():
        widx, cu = RU.get_window_index(grid, window_size=112, spatial_merge_size=2, patch_size=14)
        out[f"{name}/window_index"] = widx.numpy()
        out[f"{name}/cu_seqlens"] = cu.numpy()
        out[f"{name}/grid"] = np.asarray(grid, dtype=np.int64)
        for hd in (80, 64):
            cos, sin = R.compute_rope_2d(grid, head_dim=hd, spatial_merge_size=2, theta=10000.0,
                                         device="cpu", dtype=torch.float32)
            out[f"{name}/cos{hd}"] = cos.numpy()
            out[f"{name}/sin{hd}"] = sin.numpy()
            cosw, sinw = R.compute_rope_2d(grid, head_dim=hd, spatial_merge_size=2, theta=10000.0,
                                           device="cpu", dtype=torch.float32, window_idx=widx)
            out[f"{name}/cos{hd}_win"] = cosw.numpy()
            out[f"{name}/sin{hd}_win"] = sinw.numpy()
        cosb, _ = R.compute_rope_2d(grid, head_dim=80, spatial_merge_size=2, theta=10000.0,
                                    device="cpu", dtype=torch.bfloat16)
        out[f"{name}/cos80_bf16_bits"] = cosb.view(torch.int16).numpy()
        T = int(sum(t * h * w for t, h, w in grid))
        x = torch.arange(T * 3, dtype=torch.float32).reshape(T, 3)
        xs = RU.window_shuffle(x, widx, spatial_merge_size=2)
        out[f"{name}/shuffled"] = xs.numpy()
        out[f"{name}/unshuffled"] = RU.window_unshuffle(xs, widx, spatial_merge_size=2).numpy()
    np.savez_compressed(os.path.join(HERE, "golden_host.npz"), **out)


def run_ref_kernel(q, k, v, cos, sin, cu, block_m=64, block_n=64):
    T, H, D = q.shape
    out = torch.empty_like(q)
    cu = cu.to(torch.int32)
    nwin = cu.numel() - 1
    max_len = int((cu[1:] - cu[:-1]).max())
    grid = (-(-max_len // block_m), nwin * H)
    R.fused_attn_kernel.fn[grid](
        q, k, v, cos, sin, out, cu,
        q.stride(0), q.stride(1), q.stride(2),
        k.stride(0), k.stride(1), k.stride(2),
        v.stride(0), v.stride(1), v.stride(2),
        cos.stride(0), cos.stride(1),
        out.stride(0), out.stride(1), out.stride(2),
        nwin, H, max_len,
        HEAD_DIM=D, HEAD_DIM_PADDED=R.next_pow2(D), HALF_DIM_PADDED=R.next_pow2(D // 2),
        BLOCK_M=block_m, BLOCK_N=block_n,
    )
    return out


KERNEL_CASES = [
    # name, grid, windowed, heads, dtype, head_dim
    ("win16x16_f16", [(1, 16, 16)], True, 2, torch.float16, 80),
    ("win12x20_f16", [(1, 12, 20)], True, 2, torch.float16, 80),
    ("full16x16_f16", [(1, 16, 16)], False, 2, torch.float16, 80),
    ("win8x24_f32", [(1, 8, 24)], True, 2, torch.float32, 80),
    ("multi_f16", [(1, 8, 8), (1, 6, 10)], True, 1, torch.float16, 64),
    ("hd72_win16x12_f16", [(1, 16, 12)], True, 2, torch.float16, 72),  # the reference bench.py:31-34 head dim
]


def kernel_goldens():
    out = {}
    for i, (name, grid, windowed, H, dt, D) in enumerate(KERNEL_CASES):
        g = torch.Generator().manual_seed(1000 + i)
        T = int(sum(t * h * w for t, h, w in grid))
        q = torch.randn(T, H, D, generator=g).to(dt)
        k = torch.randn(T, H, D, generator=g).to(dt)
        v = torch.randn(T, H, D, generator=g).to(dt)
        if windowed:
            widx, cu = RU.get_window_index(grid, window_size=112, spatial_merge_size=2, patch_size=14)
            cos, sin = R.compute_rope_2d(grid, head_dim=D, spatial_merge_size=2, theta=10000.0,
                                         device="cpu", dtype=torch.float32, window_idx=widx)
        else:
            cu = torch.tensor([0, T], dtype=torch.int32)
            cos, sin = R.compute_rope_2d(grid, head_dim=D, spatial_merge_size=2, theta=10000.0,
                                         device="cpu", dtype=torch.float32)
        o = run_ref_kernel(q, k, v, cos, sin, cu)
        out[f"{name}/q"] = q.float().numpy() if dt == torch.float32 else q.numpy()
        out[f"{name}/k"] = k.float().numpy() if dt == torch.float32 else k.numpy()
        out[f"{name}/v"] = v.float().numpy() if dt == torch.float32 else v.numpy()
        out[f"{name}/cos"] = cos.numpy()
        out[f"{name}/sin"] = sin.numpy()
        out[f"{name}/cu_seqlens"] = cu.numpy()
        out[f"{name}/out"] = o.float().numpy() if dt == torch.float32 else o.numpy()
        print(name, T, H, D, dt, "cu", cu.tolist()[:6], "...", flush=True)
    np.savez_compressed(os.path.join(HERE, "golden_kernel.npz"), **out)


if __name__ == "__main__":
    host_goldens()
    kernel_goldens()
    print("wrote", os.listdir(HERE))
