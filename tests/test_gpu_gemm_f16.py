"""Dense fp16 GEMM on the tcgen05 tensor cores (mcv_gemm_f16, the M > 8 half
of matmul_b_transposed, src/csrc/lib/ops.cpp:215-322) against the CPU oracle:
fp16 outputs within |d| <= 1e-2 + 1e-3|ref|; the split-k clusters must give
the same result as a single CTA."""
import numpy as np
import pytest

import make_golden as golden
import oracle
from conftest import assert_f16_close
from mcv_b200 import synth

pytestmark = pytest.mark.gpu


def run(torch, x, w_nk):
    import mcv_b200 as mcv
    M, N = x.shape[0], w_nk.shape[0]
    out = torch.empty((M, N), dtype=torch.float16, device="cuda")
    mcv.gemm_f16(torch.from_numpy(x).cuda(), torch.from_numpy(w_nk).cuda(), out)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("M", [16, 256, 1024])
@pytest.mark.parametrize("K", [1024, 4096])
def test_gemm_vs_oracle(cuda, M, K):
    N = 3584 if K == 1024 else 1024
    r = synth.rng(M + K)
    x = r.standard_normal((M, K), dtype=np.float32).astype(np.float16)
    w = (r.standard_normal((N, K), dtype=np.float32) * 0.03).astype(np.float16)
    ref = oracle.gemv_f16(x, w, layout=0) if M <= 256 else None
    got = run(cuda, x, w)
    if ref is None:  # spot-check rows of the large case (the scalar oracle is slow)
        rows = np.array([0, 1, 255, 256, 511, 777, 1023])
        ref = oracle.gemv_f16(x[rows], w, layout=0)
        got = got[rows]
    assert_f16_close(got, ref, what=f"gemm M={M} K={K}")


@pytest.mark.parametrize("M,K,N", [(9, 128, 40), (100, 192, 136), (300, 512, 520), (17, 64, 8), (33, 256, 1000)])
def test_ragged_shapes(cuda, M, K, N):
    r = synth.rng(M * 3 + N)
    x = r.standard_normal((M, K), dtype=np.float32).astype(np.float16)
    w = (r.standard_normal((N, K), dtype=np.float32) * 0.05).astype(np.float16)
    assert_f16_close(run(cuda, x, w), oracle.gemv_f16(x, w, layout=0), what=f"gemm {M}x{K}x{N}")


def test_split_k_matches_single_cta(cuda):
    import mcv_b200 as mcv
    torch = cuda
    r = synth.rng(5)
    x = torch.from_numpy(r.standard_normal((32, 4096), dtype=np.float32).astype(np.float16)).cuda()
    w = torch.from_numpy((r.standard_normal((1024, 4096), dtype=np.float32) * 0.03).astype(np.float16)).cuda()
    outs = []
    for split in (1, 2, 4, 8):
        mcv.set_tuning(5, split)
        o = torch.empty((32, 1024), dtype=torch.float16, device="cuda")
        mcv.gemm_f16(x, w, o)
        torch.cuda.synchronize()
        outs.append(o.cpu().numpy().astype(np.float32))
    mcv.set_tuning(5, 0)
    ref = oracle.gemv_f16(x.cpu().numpy(), w.cpu().numpy(), layout=0)
    for o in outs:
        assert_f16_close(o, ref, what="split-k")
    assert mcv.device_errors() == 0


def test_matmul_b_transposed_prefill_golden(cuda):
    """tests/test_matmul.cpp's M=89 case shape through matmul_b_transposed
    (M > 8 -> the tensor-core GEMM), weights transposed on the GPU."""
    import mcv_b200 as mcv
    torch = cuda
    x = golden.load("matmul_1x1024x4096.x")
    w_kn = golden.load("matmul_1x1024x4096.w_kn")
    xs = np.repeat(x, 89, axis=0).view(np.float16)
    w_nk = torch.empty((4096, 1024), dtype=torch.float16, device="cuda")
    mcv.transpose_f16(torch.from_numpy(w_kn.view(np.float16)).cuda(), w_nk)
    out = torch.empty((89, 4096), dtype=torch.float16, device="cuda")
    mcv.matmul_b_transposed(torch.from_numpy(xs).cuda(), w_nk, out)
    torch.cuda.synchronize()
    ref = np.repeat(golden.load("matmul_1x1024x4096.ref"), 89, axis=0)
    assert_f16_close(out.cpu().numpy(), ref, what="prefill golden")
    assert np.array_equal(w_nk.cpu().numpy().view(np.uint16), np.ascontiguousarray(w_kn.T))
