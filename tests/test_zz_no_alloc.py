"""frattn_fwd_noalloc: the allocation-free entry point, called through the C ABI.

This entry point serves callers that cannot allocate device memory when they
call attention, for example a plugin running inside another framework that
owns the allocator, or a serving loop where cudaMalloc would stall the device.
Its work list lives in a fixed array inside the library instead of a
caller-provided workspace. The test checks that two calls in a row give the
output of the regular entry point (frattn_fwd with its own workspace), within
the parity tolerance used everywhere else. The second call covers state left
behind by the first call in the shared array.

The file name makes pytest collect it last.
"""
import pytest
import torch

from fused_rope_attn_b200 import _lib, fused_rope_attention, last_status
from gpu_cases import cu_case

pytestmark = pytest.mark.gpu
DEV = "cuda"


def call_noalloc(q, k, v, cos, sin, cu, out, status):
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    return lib.frattn_fwd_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), cos.data_ptr(), sin.data_ptr(), _lib.F32,
        cu.data_ptr(), cu.numel() - 1, q.shape[0], q.shape[1], q.shape[2], 0, _lib.BF16,
        out.data_ptr(), status.data_ptr(), stream)


def test_noalloc_matches_regular_entry_point_twice():
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    # Two different segmentations so the second call sees a different work list
    # than the one the first call left in the shared array.
    for seed, cu_list in ((1, [0, 64, 128, 330, 331, 700]), (2, [0, 40, 900, 964, 1000])):
        q, k, v, cos, sin, cu = (t.to(DEV) for t in cu_case(cu_list, H=4, seed=seed))
        ref = fused_rope_attention(q, k, v, cos, sin, cu)
        out = torch.full_like(q, float("nan"))
        assert call_noalloc(q, k, v, cos, sin, cu, out, status) == 0
        torch.cuda.synchronize()
        assert int(status.item()) == 0 and last_status() == 0
        err = (out.float() - ref.float()).abs()
        assert torch.isfinite(out.float()).all()
        assert err.max().item() <= 2e-2 and err.mean().item() <= 2e-3


def test_noalloc_small_long_segment_matches_oracle():
    # Few tokens but one segment longer than a 128-row tile: the case where a
    # rotated-K copy would fit into the library's array. It must not be placed
    # there (every rotation stays in the attention kernel); the output is
    # checked directly against the CPU oracle, twice in a row.
    from oracle import rope_attn_oracle as O
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    q, k, v, cos, sin, cu = cu_case([0, 256], H=1, D=64, seed=11)
    want = O.rope_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), cos.numpy(), sin.numpy(),
                            cu.numpy())
    qd, kd, vd, cd, sd, cud = (t.to(DEV) for t in (q, k, v, cos, sin, cu))
    for _ in range(2):
        out = torch.full_like(qd, float("nan"))
        assert call_noalloc(qd, kd, vd, cd, sd, cud, out, status) == 0
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        err = (out.float().cpu() - torch.from_numpy(want)).abs()
        assert err.max().item() <= 2e-2 and err.mean().item() <= 2e-3


def test_noalloc_rejects_more_tokens_than_its_array_holds():
    q = torch.zeros(16, 1, 80, dtype=torch.bfloat16, device=DEV)
    lib = _lib.load()
    rc = lib.frattn_fwd_noalloc(q.data_ptr(), q.data_ptr(), q.data_ptr(), q.data_ptr(), q.data_ptr(), _lib.F32,
                                q.data_ptr(), 1, _lib.NOALLOC_MAX_TOKENS + 1, 1, 80, 0, _lib.BF16,
                                q.data_ptr(), None, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.E_NOALLOC_LIMIT
