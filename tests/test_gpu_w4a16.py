"""W4A16 GEMV parity on the GPU (through the C ABI) against the CPU oracle and
the reference test's golden outputs.  Tolerance (fp16 outputs):
|got - ref| <= 1e-2 + 1e-3 * |ref|."""
import numpy as np
import pytest

import make_golden as golden
import oracle
from conftest import assert_f16_close
from mcv_b200 import synth

pytestmark = pytest.mark.gpu


def run_gemv(torch, x, w):
    import mcv_b200
    xd = torch.from_numpy(np.ascontiguousarray(x).view(np.float16)).cuda()
    out = torch.empty((xd.shape[0], w.N), dtype=torch.float16, device="cuda")
    mcv_b200.matmul_w4a16(xd, w, out)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_reference_test_golden(cuda):
    # tests/test_matmul_w4a16.cpp inputs: signed int8 weights in [-8,7] with
    # no zeros == q = w + 8 with zero 8
    import mcv_b200
    x = golden.load("w4a16.x")
    w = golden.load("w4a16.w")
    s = golden.load("w4a16.s")
    q = (w.astype(np.int16) + 8).astype(np.uint8)
    z = np.full((8, 3584), 8, np.uint8)
    dw = mcv_b200.pack_w4a16(q, z, s)
    out = run_gemv(cuda, x, dw)
    assert_f16_close(out, golden.load("w4a16.ref"), what="golden w4a16")
    # the reference test's own pass criterion: no |d| > 0.1
    assert np.max(np.abs(out.astype(np.float32) - golden.load("w4a16.ref"))) <= 0.1


def test_constant_known_answer(cuda):
    import mcv_b200
    q = np.full((1024, 3584), 9, np.uint8)
    z = np.full((8, 3584), 8, np.uint8)
    s = golden.load("w4a16_const.s")
    out = run_gemv(cuda, golden.load("w4a16_const.x"), mcv_b200.pack_w4a16(q, z, s))
    assert np.all(out == np.float16(1024.0))


@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 8])
def test_config0_all_m(cuda, M):
    import mcv_b200
    x, q, z, s = synth.w4a16_inputs(M, 1024, 3584, seed=M)
    ref = oracle.w4a16_gemv(x, oracle.w4a16_fold_zeros(q, z), s, nthreads=8)
    out = run_gemv(cuda, x, mcv_b200.pack_w4a16(q, z, s))
    assert_f16_close(out, ref, what=f"config0 M={M}")


@pytest.mark.parametrize("K,N", [(1024, 16), (1024, 512), (1024, 6144), (2048, 1024), (3584, 1024),
                                 (4096, 4096), (1024, 100), (128, 8), (8192, 64), (384, 40), (1152, 24)])
def test_shapes(cuda, K, N):
    import mcv_b200
    x, q, z, s = synth.w4a16_inputs(1, K, N, seed=K * 7 + N)
    ref = oracle.w4a16_gemv(x, oracle.w4a16_fold_zeros(q, z), s, nthreads=8)
    out = run_gemv(cuda, x, mcv_b200.pack_w4a16(q, z, s))
    assert_f16_close(out, ref, what=f"K={K} N={N}")


def test_gptq_awq_and_tile_inputs(cuda):
    import mcv_b200
    K, N = 1024, 3584
    x, q, _, s = synth.w4a16_inputs(2, K, N, seed=21)
    r = synth.rng(22)
    zg = r.integers(1, 17, (K // 128, N), dtype=np.uint8)   # GPTQ true zeros 1..16
    qw, qz = synth.gptq_pack(q, zg)
    gidx = (np.arange(K) // 128).astype(np.int32)
    wg = oracle.unpack_gptq(qw, qz, gidx, K // 128)
    out = run_gemv(cuda, x, mcv_b200.pack_w4a16_gptq(qw, qz, gidx, s))
    assert_f16_close(out, oracle.w4a16_gemv(x, wg, s, nthreads=8), what="gptq")

    za = r.integers(0, 16, (K // 128, N), dtype=np.uint8)
    aw, az = synth.awq_pack(q, za)
    wa = oracle.unpack_awq(aw, az)
    out = run_gemv(cuda, x, mcv_b200.pack_w4a16_awq(aw, az, s))
    assert_f16_close(out, oracle.w4a16_gemv(x, wa, s, nthreads=8), what="awq")

    tiles = oracle.w4a16_pack_tiles(wg)
    out = run_gemv(cuda, x, mcv_b200.pack_w4a16_from_tiles(tiles, s, K, N))
    assert_f16_close(out, oracle.w4a16_gemv(x, wg, s, nthreads=8), what="reference tiles")


def test_deterministic_and_pdl_off(cuda):
    import mcv_b200
    x, q, z, s = synth.w4a16_inputs(1, 1024, 3584, seed=5)
    w = mcv_b200.pack_w4a16(q, z, s)
    a = run_gemv(cuda, x, w)
    b = run_gemv(cuda, x, w)
    mcv_b200.set_pdl(False)
    try:
        c = run_gemv(cuda, x, w)
    finally:
        mcv_b200.set_pdl(True)
    assert np.array_equal(a.view(np.uint16), b.view(np.uint16))
    assert np.array_equal(a.view(np.uint16), c.view(np.uint16))


def test_chained_gemvs_under_pdl(cuda):
    """A dependent chain (output of one GEMV is the next one's input), all on
    one stream with programmatic dependent launch, matches step-by-step."""
    import mcv_b200
    torch = cuda
    dims = [1024, 3584, 1024, 2048, 1024]
    ws, host = [], []
    for i in range(len(dims) - 1):
        x, q, z, s = synth.w4a16_inputs(1, dims[i], dims[i + 1], seed=100 + i)
        s = (s.astype(np.float32) * 0.05).astype(np.float16)  # keep activations O(1)
        ws.append(mcv_b200.pack_w4a16(q, z, s))
        host.append((q, z, s))
    x0 = synth.w4a16_inputs(1, 1024, 8, seed=99)[0]
    bufs = [torch.from_numpy(x0.copy()).cuda()] + [torch.empty((1, d), dtype=torch.float16, device="cuda")
                                                   for d in dims[1:]]
    for i, w in enumerate(ws):
        mcv_b200.matmul_w4a16(bufs[i], w, bufs[i + 1])
    torch.cuda.synchronize()
    cur = x0
    for i, (q, z, s) in enumerate(host):
        got = bufs[i + 1].cpu().numpy()
        ref = oracle.w4a16_gemv(cur, oracle.w4a16_fold_zeros(q, z), s, nthreads=8)
        assert_f16_close(got, ref, what=f"chain step {i}")
        cur = got  # next step consumes exactly what the GPU produced


@pytest.mark.parametrize("M", [1, 3, 8])
def test_grouped_mixed_problems(cuda, M):
    """One grouped launch over problems of different K/N (a linear-attention
    layer's same-input projections plus unrelated ones), each checked alone."""
    import mcv_b200
    torch = cuda
    shapes = [(1024, 6144), (1024, 2048), (1024, 16), (1024, 16), (2048, 1024), (3584, 1024), (1024, 100)]
    items, refs = [], []
    for i, (K, N) in enumerate(shapes):
        x, q, z, s = synth.w4a16_inputs(M, K, N, seed=300 + i)
        w = mcv_b200.pack_w4a16(q, z, s)
        out = torch.empty((M, N), dtype=torch.float16, device="cuda")
        items.append((torch.from_numpy(x).cuda(), w, out))
        refs.append(oracle.w4a16_gemv(x, oracle.w4a16_fold_zeros(q, z), s, nthreads=8))
    mcv_b200.matmul_w4a16_grouped(items, M=M)
    torch.cuda.synchronize()
    for (x, w, out), ref, (K, N) in zip(items, refs, shapes):
        assert_f16_close(out.cpu().numpy(), ref, what=f"grouped K={K} N={N}")


def test_grouped_more_than_one_launch(cuda):
    import mcv_b200
    torch = cuda
    x, q, z, s = synth.w4a16_inputs(1, 1024, 512, seed=400)
    w = mcv_b200.pack_w4a16(q, z, s)
    xd = torch.from_numpy(x).cuda()
    outs = [torch.empty((1, 512), dtype=torch.float16, device="cuda") for _ in range(100)]
    mcv_b200.matmul_w4a16_grouped([(xd, w, o) for o in outs])
    torch.cuda.synchronize()
    ref = oracle.w4a16_gemv(x, oracle.w4a16_fold_zeros(q, z), s)
    first = outs[0].cpu().numpy()
    assert_f16_close(first, ref, what="grouped x100")
    for o in outs[1:]:
        assert np.array_equal(o.cpu().numpy().view(np.uint16), first.view(np.uint16))


@pytest.mark.parametrize("mode", [1, 2, 3])
@pytest.mark.parametrize("M,K,N", [(1, 1024, 3584), (3, 3584, 1024), (8, 384, 200), (2, 8192, 64)])
def test_both_kernels_agree(cuda, mode, M, K, N):
    """Both streaming kernels (modes 1, 3) and the K-split kernel (mode 2)."""
    import mcv_b200
    x, q, z, s = synth.w4a16_inputs(M, K, N, seed=K + N + M)
    w = mcv_b200.pack_w4a16(q, z, s)
    ref = oracle.w4a16_gemv(x, oracle.w4a16_fold_zeros(q, z), s, nthreads=8)
    mcv_b200.set_tuning(mcv_b200.TUNE_W4A16_MODE, mode)
    try:
        out = run_gemv(cuda, x, w)
    finally:
        mcv_b200.set_tuning(mcv_b200.TUNE_W4A16_MODE, 0)
    assert_f16_close(out, ref, what=f"mode={mode}")


def test_grouped_tma_many_problems(cuda):
    """Enough problems that the default picks the bulk-copy streaming kernel,
    mixed K (several 512-k chunks per strip) and a ragged N."""
    import mcv_b200
    torch = cuda
    items, refs = [], []
    for i in range(40):
        K, N = ((1024, 3584), (3584, 1024), (2048, 1000))[i % 3]
        x, q, z, s = synth.w4a16_inputs(2, K, N, seed=600 + i)
        w = mcv_b200.pack_w4a16(q, z, s)
        items.append((torch.from_numpy(x).cuda(), w, torch.empty((2, N), dtype=torch.float16, device="cuda")))
        if i < 6:
            refs.append(oracle.w4a16_gemv(x, oracle.w4a16_fold_zeros(q, z), s, nthreads=8))
    mcv_b200.matmul_w4a16_grouped(items, M=2)
    torch.cuda.synchronize()
    for (x, w, out), ref in zip(items, refs):
        assert_f16_close(out.cpu().numpy(), ref, what=f"tma grouped K={w.K} N={w.N}")


def test_no_device_errors_recorded(cuda):
    """No bounded wait in any W4A16 kernel gave up during the tests above."""
    import mcv_b200
    assert mcv_b200.device_errors() == 0


@pytest.mark.parametrize("M,K,N", [(9, 1024, 3584), (16, 1024, 4096), (24, 3584, 1024), (32, 1024, 3584),
                                   (13, 8192, 64), (32, 128, 40), (33, 1024, 520), (48, 2048, 1024),
                                   (64, 1024, 3584), (57, 8192, 40)])
def test_batched_decode_gemv(cuda, M, K, N):
    """M = 9..64 on the widened GEMV (one dequantised fragment, up to eight MMAs)."""
    import mcv_b200
    x, q, z, s = synth.w4a16_inputs(M, K, N, seed=M * 100 + K)
    ref = oracle.w4a16_gemv(x, oracle.w4a16_fold_zeros(q, z), s, nthreads=8)
    out = run_gemv(cuda, x, mcv_b200.pack_w4a16(q, z, s))
    assert_f16_close(out, ref, what=f"batched M={M} K={K} N={N}")
