"""W8A8 on the GPU vs the CPU oracle: int8 quantized activations, int32
accumulators and fp16 outputs must all be BIT-EXACT (the float steps use
explicitly rounded fp32 operations in the same order as the reference)."""
import numpy as np
import pytest

import make_golden as golden
import oracle
from mcv_b200 import synth

pytestmark = pytest.mark.gpu


def D(torch, a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.float16)
    return torch.from_numpy(a).cuda()


def H(t):
    a = t.cpu().numpy()
    return a.view(np.uint16) if a.dtype == np.float16 else a


@pytest.mark.parametrize("layout", [1, 0])
def test_i32_golden(cuda, layout):
    import mcv_b200
    torch = cuda
    x = golden.load("w8a8_i32.x")
    w = golden.load("w8a8_i32.w")
    wl = w if layout == 1 else np.ascontiguousarray(w.T)
    acc = torch.empty((1, 3584), dtype=torch.int32, device="cuda")
    mcv_b200.matmul_w8a8_i32(D(torch, x), D(torch, wl), acc, w_layout=layout)
    torch.cuda.synchronize()
    assert np.array_equal(H(acc), golden.load("w8a8_i32.ref"))


def test_dequant_golden(cuda):
    import mcv_b200
    torch = cuda
    acc = golden.load("w8a8_dequant.acc")
    xs = golden.load("w8a8_dequant.xs")
    ws = golden.load("w8a8_dequant.ws")
    out = torch.empty((1, 3584), dtype=torch.float16, device="cuda")
    mcv_b200.w8a8_dequant(D(torch, acc), D(torch, xs), D(torch, ws), out)
    torch.cuda.synchronize()
    assert np.array_equal(H(out), oracle.w8a8_dequant(acc, xs, ws))
    assert np.max(np.abs(H(out).view(np.float16).astype(np.float32) - golden.load("w8a8_dequant.ref"))) < 0.02


@pytest.mark.parametrize("M", [1, 4, 8])
def test_quantize_exact(cuda, M):
    import mcv_b200
    torch = cuda
    x, _, _ = synth.w8a8_inputs(M, 1024, 16, seed=M)
    x[0, :7] = np.float16([0.5, -0.5, 1e-4, -65504, 3.0, 0, -0.0])  # clamp / rounding edges
    xq = torch.empty((M, 1024), dtype=torch.int8, device="cuda")
    xs = torch.empty(M, dtype=torch.float16, device="cuda")
    mcv_b200.w8a8_quantize(D(torch, x), xq, xs)
    torch.cuda.synchronize()
    rq, rs = oracle.w8a8_quantize(x)
    assert np.array_equal(H(xq), rq)
    assert np.array_equal(H(xs), rs)
    z = torch.zeros((1, 256), dtype=torch.float16, device="cuda")
    xq0 = torch.empty((1, 256), dtype=torch.int8, device="cuda")
    xs0 = torch.empty(1, dtype=torch.float16, device="cuda")
    mcv_b200.w8a8_quantize(z, xq0, xs0)
    torch.cuda.synchronize()
    assert np.all(H(xq0) == 0) and H(xs0)[0] == oracle.w8a8_quantize(np.zeros((1, 256), np.float16))[1][0]


@pytest.mark.parametrize("M", [1, 4, 8])
@pytest.mark.parametrize("N", [1024, 3584])
@pytest.mark.parametrize("layout", [0, 1])
def test_fused_config2_exact(cuda, M, N, layout):
    import mcv_b200
    torch = cuda
    K = 1024
    x, w, ws = synth.w8a8_inputs(M, K, N, seed=M * 100 + N)
    racc, rout = oracle.w8a8_fused(x, w, ws, nthreads=8)
    rq, rs = oracle.w8a8_quantize(x)
    wl = np.ascontiguousarray(w.T) if layout == 0 else w
    out = torch.empty((M, N), dtype=torch.float16, device="cuda")
    acc = torch.empty((M, N), dtype=torch.int32, device="cuda")
    xq = torch.empty((M, K), dtype=torch.int8, device="cuda")
    xs = torch.empty(M, dtype=torch.float16, device="cuda")
    mcv_b200.w8a8_fused(D(torch, x), D(torch, wl), D(torch, ws), out, acc, xq, xs, w_layout=layout)
    torch.cuda.synchronize()
    assert np.array_equal(H(acc), racc)
    assert np.array_equal(H(out), rout)
    assert np.array_equal(H(xq), rq)
    assert np.array_equal(H(xs), rs)
    if layout == 0:  # optional intermediates may be omitted on the fast path
        out2 = torch.empty((M, N), dtype=torch.float16, device="cuda")
        mcv_b200.w8a8_fused(D(torch, x), D(torch, wl), D(torch, ws), out2, w_layout=0)
        torch.cuda.synchronize()
        assert np.array_equal(H(out2), rout)


@pytest.mark.parametrize("K,N", [(1024, 3584), (2048, 1024), (4096, 16), (16, 48)])
def test_gemm_shapes_exact(cuda, K, N):
    import mcv_b200
    torch = cuda
    r = synth.rng(K + N)
    M = 3
    xq = r.integers(-128, 128, (M, K), dtype=np.int8)
    w = r.integers(-128, 128, (K, N), dtype=np.int8)
    ref = oracle.w8a8_gemm_i32(xq, w)
    for layout, wl in ((1, w), (0, np.ascontiguousarray(w.T))):
        acc = torch.empty((M, N), dtype=torch.int32, device="cuda")
        mcv_b200.matmul_w8a8_i32(D(torch, xq), D(torch, wl), acc, w_layout=layout)
        torch.cuda.synchronize()
        assert np.array_equal(H(acc), ref), layout


@pytest.mark.parametrize("layout", [0, 1])
def test_quantize_weight_exact(cuda, layout):
    import mcv_b200
    torch = cuda
    r = synth.rng(31)
    K, N = 1024, 512
    w = (r.standard_normal((K, N), dtype=np.float32) * 0.03).astype(np.float16)
    w[:, 7] = 0  # all-zero column -> scale clamps to 1e-8
    rq, rs = oracle.quantize_dense_weight_w8a8(w)
    wq = torch.empty((N, K) if layout == 0 else (K, N), dtype=torch.int8, device="cuda")
    sc = torch.empty(N, dtype=torch.float16, device="cuda")
    mcv_b200.quantize_dense_weight_w8a8(D(torch, w), wq, sc, w_layout=layout)
    torch.cuda.synchronize()
    got = H(wq) if layout == 1 else H(wq).T
    assert np.array_equal(got, rq)
    assert np.array_equal(H(sc), rs)


@pytest.mark.parametrize("M", [1, 2, 3, 5, 8])
def test_dp4a_and_tensor_core_kernels_same_bits(cuda, M):
    """The DP4A and the mma.sync s8 kernels give the same int32 sums and the
    same fp16 outputs (integer sums are exact in any order)."""
    import mcv_b200 as mcv
    torch = cuda
    K, N = 2048, 520
    x, w8, ws8 = synth.w8a8_inputs(M, K, N, seed=40 + M)
    xd = torch.from_numpy(x).cuda()
    wt = torch.from_numpy(np.ascontiguousarray(w8.T)).cuda()
    wsd = torch.from_numpy(ws8).cuda()
    got = {}
    for kern in (1, 2):
        mcv.set_tuning(mcv.TUNE_W8A8_KERNEL, kern)
        try:
            out = torch.empty((M, N), dtype=torch.float16, device="cuda")
            acc = torch.empty((M, N), dtype=torch.int32, device="cuda")
            mcv.w8a8_fused(xd, wt, wsd, out, acc=acc, w_layout=0)
            torch.cuda.synchronize()
            got[kern] = (out.cpu().numpy().view(np.uint16), acc.cpu().numpy())
        finally:
            mcv.set_tuning(mcv.TUNE_W8A8_KERNEL, 0)
    assert np.array_equal(got[1][1], got[2][1])
    assert np.array_equal(got[1][0], got[2][0])
    _, r8 = oracle.w8a8_fused(x, w8, ws8)
    assert np.array_equal(got[2][0], r8)


def test_gpu_weight_quantizer_equals_reference_code_output(cuda):
    """The GPU quantizer against the reference's own quantize_dense_weight_w8a8
    (src/csrc/lib/quantized_weight.cpp:231-268), run on the CPU by
    tests/golden/make_ref_fixtures.py: int8 weights and fp16 scales bit-exact,
    including a zero column and a column with a 65000 outlier."""
    import make_ref_fixtures as reffix
    import mcv_b200 as mcv
    torch = cuda
    w = reffix.w8a8_quant_input()
    ref_wq, ref_ws = reffix.load_w8a8_quant()
    K, N = w.shape
    wq = torch.empty((K, N), dtype=torch.int8, device="cuda")
    ws = torch.empty(N, dtype=torch.float16, device="cuda")
    mcv.quantize_dense_weight_w8a8(torch.from_numpy(w).cuda(), wq, ws, w_layout=1)
    torch.cuda.synchronize()
    assert np.array_equal(wq.cpu().numpy(), ref_wq)
    assert np.array_equal(ws.cpu().numpy().view(np.uint16), ref_ws)


@pytest.mark.parametrize("M,N", [(1, 3584), (4, 1024), (8, 3584)])
def test_prequant_gemv_equals_fused(cuda, M, N):
    """matmul_decode_w8a8_prequant: quantize once, then int32 GEMV + dequant in
    one kernel; bit-exact against the oracle and the one-kernel fused path."""
    import mcv_b200 as mcv
    torch = cuda
    x, w, ws = synth.w8a8_inputs(M, 1024, N, seed=M * 7 + N)
    xd = torch.from_numpy(x).cuda()
    wt = torch.from_numpy(np.ascontiguousarray(w.T)).cuda()
    wsd = torch.from_numpy(ws).cuda()
    xq = torch.empty((M, 1024), dtype=torch.int8, device="cuda")
    xs = torch.empty(M, dtype=torch.float16, device="cuda")
    mcv.w8a8_quantize(xd, xq, xs)
    out = torch.empty((M, N), dtype=torch.float16, device="cuda")
    acc = torch.empty((M, N), dtype=torch.int32, device="cuda")
    for kernel in (1, 2):  # DP4A and the integer tensor cores
        mcv.set_tuning(6, kernel)
        out.fill_(0)
        mcv.matmul_decode_w8a8_prequant(xq, xs, wt, wsd, out, acc=acc)
        torch.cuda.synchronize()
        r_acc, r_out = oracle.w8a8_fused(x, w, ws)
        assert np.array_equal(acc.cpu().numpy(), np.asarray(r_acc).reshape(M, N))
        assert np.array_equal(out.cpu().numpy().view(np.uint16), np.asarray(r_out).reshape(M, N))
    mcv.set_tuning(6, 0)


@pytest.mark.parametrize("M", [1, 4])
def test_grouped_fused_equals_single(cuda, M):
    """Several fused W8A8 GEMVs in one launch (e.g. gate and up on one input):
    each bit-exact against the oracle."""
    import mcv_b200 as mcv
    torch = cuda
    items, refs = [], []
    x, _, _ = synth.w8a8_inputs(M, 1024, 16, seed=90 + M)
    xd = torch.from_numpy(x).cuda()
    for i, N in enumerate((3584, 3584, 1024, 40)):
        _, w, ws = synth.w8a8_inputs(M, 1024, N, seed=100 * M + i)
        out = torch.zeros((M, N), dtype=torch.float16, device="cuda")
        items.append((xd, torch.from_numpy(np.ascontiguousarray(w.T)).cuda(), torch.from_numpy(ws).cuda(), out))
        refs.append(np.asarray(oracle.w8a8_fused(x, w, ws)[1]).reshape(M, N))
    mcv.w8a8_fused_grouped(items)
    torch.cuda.synchronize()
    for (_, _, _, out), ref in zip(items, refs):
        assert np.array_equal(out.cpu().numpy().view(np.uint16), ref)
