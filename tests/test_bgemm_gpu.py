"""Batched projections on the tensor cores (infernt_bgemm_bf16) against a
plain PyTorch FP32 matmul of the same bf16 operands.

The partials of the K splits are added in split order on the host side of
the test; the tolerance allows for FP32 accumulation in a different order:
max-abs error <= 2e-5 of the largest |Y| plus 1e-6."""
import pytest

import infernt_b200 as ib

pytestmark = pytest.mark.gpu


def _torch():
    import torch
    return torch


def run_bgemm(N, K, T, splits, seed=0):
    torch = _torch()
    g = torch.Generator(device="cuda").manual_seed(seed)
    W = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    X = torch.randn(T, K, device="cuda", generator=g).to(torch.bfloat16)
    part = torch.full((splits, T, N), float("nan"), device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ib.call("infernt_bgemm_bf16", W.data_ptr(), N, K, X.data_ptr(), T, part.data_ptr(), splits, err.data_ptr(),
            torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    got = part[0].clone()
    for s in range(1, splits):
        got += part[s]
    want = X.float() @ W.float().t()
    return got, want


@pytest.mark.parametrize("N,K,T,splits", [
    (128, 64, 1, 1),          # one tile, one stage
    (256, 512, 16, 2),
    (2560, 2048, 64, 8),      # Q|K|V of the TinyLlama shape, 64 sequences
    (2048, 5632, 64, 11),     # down projection
    (384, 4096, 37, 16),      # token count padded to 48
    (128, 1024, 256, 4),      # the largest batch
])
def test_bgemm_matches_torch(N, K, T, splits):
    got, want = run_bgemm(N, K, T, splits)
    err = float((got - want).abs().max())
    scale = float(want.abs().max())
    assert err <= 2e-5 * scale + 1e-6, (err, scale)


def test_bgemm_rejects_bad_shapes():
    torch = _torch()
    W = torch.zeros(128, 64, dtype=torch.bfloat16, device="cuda")
    X = torch.zeros(1, 64, dtype=torch.bfloat16, device="cuda")
    part = torch.zeros(1, 1, 128, device="cuda")
    for args in [(W, 100, 64, X, 1, 1), (W, 128, 60, X, 1, 1), (W, 128, 64, X, 0, 1), (W, 128, 64, X, 1, 2)]:
        with pytest.raises(ib.InferntError):
            ib.call("infernt_bgemm_bf16", args[0].data_ptr(), args[1], args[2], args[3].data_ptr(), args[4],
                    part.data_ptr(), args[5], None, None)
