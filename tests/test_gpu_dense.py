"""Dense fp16 GEMV, fused lm_head argmax and argmax_last_dim on the GPU vs the
CPU oracle / reference golden outputs.  fp16 outputs: |d| <= 1e-2 + 1e-3|ref|;
argmax indices: exact."""
import numpy as np
import pytest

import make_golden as golden
import oracle
from conftest import assert_f16_close
from mcv_b200 import synth

pytestmark = pytest.mark.gpu


def dev(torch, a, dtype=None):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.float16)
    return torch.from_numpy(a).cuda()


def gemv(torch, x, w, layout):
    import mcv_b200
    xd, wd = dev(torch, x), dev(torch, w)
    N = w.shape[0] if layout == 0 else w.shape[1]
    out = torch.empty((xd.shape[0], N), dtype=torch.float16, device="cuda")
    mcv_b200.matmul_b_transposed(xd, wd, out)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def lm_head(torch, x, w_nk, n_offset=0, fp16_logits=False):
    import mcv_b200
    xd, wd = dev(torch, x), dev(torch, w_nk)
    M = xd.shape[0]
    ws = mcv_b200.lm_head_workspace(M)
    idx = torch.empty(M, dtype=torch.int64, device="cuda")
    key = torch.empty(M, dtype=torch.int64, device="cuda")
    mcv_b200.lm_head_argmax(xd, wd, ws, out_index=idx, out_key=key, n_offset=n_offset, fp16_logits=fp16_logits)
    torch.cuda.synchronize()
    return idx.cpu().numpy(), key.cpu().numpy().view(np.uint64), ws


def test_cube_golden(cuda):
    out = gemv(cuda, golden.load("cube.x"), golden.load("cube.w_nk"), 0)
    assert_f16_close(out, golden.load("cube.ref"), what="cube")


@pytest.mark.parametrize("tag", ["matmul_4x128x64", "matmul_1x1024x4096"])
def test_matmul_golden_natural_layout(cuda, tag):
    # [K,N] "natural" B; K=128,N=64 collides with neither disambiguation rule
    out = gemv(cuda, golden.load(tag + ".x"), golden.load(tag + ".w_kn"), 1)
    assert_f16_close(out, golden.load(tag + ".ref"), what=tag)


@pytest.mark.parametrize("M", [1, 3, 8])
@pytest.mark.parametrize("layout", [0, 1])
def test_gemv_vs_oracle(cuda, M, layout):
    r = synth.rng(M * 10 + layout)
    K, N = 1024, 3584
    x = r.standard_normal((M, K), dtype=np.float32).astype(np.float16)
    w = (r.standard_normal((N, K) if layout == 0 else (K, N), dtype=np.float32) * 0.05).astype(np.float16)
    ref = oracle.gemv_f16(x, w, layout=layout)
    assert_f16_close(gemv(cuda, x, w, layout), ref, what=f"gemv M={M} layout={layout}")


def test_lm_head_pipeline_golden(cuda):
    # tests/test_lm_head_pipeline.cpp: 4 rows, H=64, V=128, weight [H,V]
    w_nk = np.ascontiguousarray(golden.load("lm_head.w").T)
    idx, _, _ = lm_head(cuda, golden.load("lm_head.x"), w_nk)
    assert np.array_equal(idx, golden.load("lm_head.ref"))


@pytest.fixture(scope="module")
def vocab():
    x, w = synth.lm_head_inputs(1024, 248094, seed=1)
    return x, w


def test_lm_head_full_vocab(cuda, vocab):
    x, w = vocab
    ref_idx, ref_best, gap = oracle.lm_head_argmax(x, w, nthreads=8)
    assert gap[0] > 1e-4, "seed gives an ambiguous top-2; pick another"
    idx, key, ws = lm_head(cuda, x, w)
    assert idx[0] == ref_idx[0]
    assert int(key[0]) == oracle.argmax_key(float(ref_best[0]), int(ref_idx[0])) or \
        (int(key[0]) & 0xFFFFFFFF) == 0xFFFFFFFF - int(ref_idx[0])
    # the workspace counter is left at zero for the next call
    assert int(ws[:4].cpu().numpy().view(np.uint32)[0]) == 0
    idx2, _, _ = lm_head(cuda, x, w)
    assert idx2[0] == idx[0]


def test_lm_head_fp16_logits_mode(cuda, vocab):
    x, w = vocab
    ref_idx, _, gap = oracle.lm_head_argmax(x, w, fp16_logits=True, nthreads=8)
    idx, _, _ = lm_head(cuda, x, w, fp16_logits=True)
    if gap[0] > 0:
        assert idx[0] == ref_idx[0]


@pytest.mark.parametrize("shards", [2, 4, 8])
def test_lm_head_shards_combine(cuda, vocab, shards):
    """Per-shard keys (contiguous ceil(V/g) row ranges with global offsets)
    combine by max into the unsharded answer: the host side of the NCCL path."""
    x, w = vocab
    V = w.shape[0]
    per = (V + shards - 1) // shards
    keys = []
    for r in range(shards):
        a, b = r * per, min(V, (r + 1) * per)
        _, k, _ = lm_head(cuda, x, np.ascontiguousarray(w[a:b]), n_offset=a)
        keys.append(int(k[0]))
    best = max(keys)
    ref_idx, _, _ = oracle.lm_head_argmax(x, w, nthreads=8)
    assert 0xFFFFFFFF - (best & 0xFFFFFFFF) == ref_idx[0]


def test_lm_head_ties_first_max(cuda):
    r = synth.rng(3)
    K, N = 256, 5000
    x = r.standard_normal((2, K), dtype=np.float32).astype(np.float16)
    w = (r.standard_normal((N, K), dtype=np.float32) * 0.02).astype(np.float16)
    w[4000] = w[1234] = np.float16(0.5) * np.sign(x[0]).astype(np.float16)  # identical best rows
    idx, _, _ = lm_head(cuda, x, w)
    ref, _, _ = oracle.lm_head_argmax(x, w)
    assert idx[0] == 1234 and idx[0] == ref[0]
    assert idx[1] == ref[1]
    # all-zero weights: every logit is 0, the first row wins
    idx0, _, _ = lm_head(cuda, x, np.zeros((777, K), np.float16))
    assert list(idx0) == [0, 0]
    # all logits negative
    wn = -np.abs(w)
    xp = np.abs(x)
    idxn, _, _ = lm_head(cuda, xp, wn)
    refn, _, _ = oracle.lm_head_argmax(xp, wn)
    assert np.array_equal(idxn, refn)


@pytest.mark.parametrize("M,K,N", [(1, 1024, 1), (1, 8, 3), (3, 2048, 33333), (8, 1024, 4096)])
def test_lm_head_shapes(cuda, M, K, N):
    r = synth.rng(M + K + N)
    x = r.standard_normal((M, K), dtype=np.float32).astype(np.float16)
    w = (r.standard_normal((N, K), dtype=np.float32) * 0.02).astype(np.float16)
    ref, _, gap = oracle.lm_head_argmax(x, w, nthreads=8)
    idx, _, _ = lm_head(cuda, x, w)
    for m in range(M):
        if gap[m] > 1e-4 or N == 1:
            assert idx[m] == ref[m], (m, idx[m], ref[m], gap[m])


def test_argmax_last_dim(cuda):
    import mcv_b200
    torch = cuda
    r = synth.rng(9)
    logits = r.standard_normal((4, 50000), dtype=np.float32).astype(np.float16)
    logits[2, 77] = logits[2, 900] = np.float16(60000)  # tie -> first
    ld = torch.from_numpy(logits).cuda()
    out = torch.empty(4, dtype=torch.int64, device="cuda")
    mcv_b200.argmax_last_dim(ld, out)
    torch.cuda.synchronize()
    assert out.cpu().tolist() == np.argmax(logits.astype(np.float32), axis=1).tolist()
    assert out[2].item() == 77


def test_lm_head_greedy_host_round_trip(cuda):
    """Host x in, host index out in one call: the same index as the device
    entry point, on two calls in a row (the workspace stays usable)."""
    import mcv_b200 as mcv
    torch = cuda
    K, V = 1024, 20000
    g = torch.Generator(device="cuda")
    g.manual_seed(21)
    w = (torch.randn((V, K), device="cuda", generator=g) * 0.02).half()
    ws = mcv.lm_head_workspace(1)
    idx_dev = torch.empty(1, dtype=torch.int64, device="cuda")
    for seed in (1, 2):
        x = torch.randn((1, K), generator=torch.Generator().manual_seed(seed)).half().pin_memory()
        x_dev = torch.empty((1, K), dtype=torch.float16, device="cuda")
        got = torch.full((1,), -7, dtype=torch.int64).pin_memory()
        mcv.lm_head_greedy_host(x, x_dev, w, idx_dev, got, ws)
        ref = torch.empty(1, dtype=torch.int64, device="cuda")
        mcv.lm_head_argmax(x.cuda(), w, ws, out_index=ref)
        torch.cuda.synchronize()
        assert int(got[0]) == int(ref.item())
        assert 0 <= int(got[0]) < V


def test_lm_head_greedy_step_prepared(cuda):
    """The prepared per-token call gives the same indices as the plain call,
    also after switching the weight between calls."""
    import mcv_b200 as mcv
    torch = cuda
    K, V = 1024, 12000
    g = torch.Generator(device="cuda")
    g.manual_seed(22)
    ws_ = [(torch.randn((V, K), device="cuda", generator=g) * 0.02).half() for _ in range(2)]
    work = mcv.lm_head_workspace(1)
    idx_dev = torch.empty(1, dtype=torch.int64, device="cuda")
    x = torch.randn((1, K), generator=torch.Generator().manual_seed(5)).half().pin_memory()
    x_dev = torch.empty((1, K), dtype=torch.float16, device="cuda")
    got = torch.full((1,), -7, dtype=torch.int64).pin_memory()
    step = mcv.LmHeadGreedyStep(x, x_dev, ws_[0], idx_dev, got, work)
    for w in (ws_[0], ws_[1], ws_[0]):
        step(w)
        ref = torch.full((1,), -9, dtype=torch.int64).pin_memory()
        mcv.lm_head_greedy_host(x, x_dev, w, idx_dev, ref, work)
        assert int(got[0]) == int(ref[0]) and 0 <= int(got[0]) < V


def test_lm_head_greedy_host_refuses_device_x(cuda):
    """x_host is read on the host: device memory there is refused with a
    status instead of faulting the process."""
    import ctypes
    import mcv_b200 as mcv
    torch = cuda
    L = mcv.lib()
    xd = torch.zeros((1, 1024), dtype=torch.float16, device="cuda")
    w = torch.zeros((64, 1024), dtype=torch.float16, device="cuda")
    ws = mcv.lm_head_workspace(1)
    idx = torch.empty(1, dtype=torch.int64, device="cuda")
    host_idx = torch.empty(1, dtype=torch.int64).pin_memory()
    st = L.mcv_lm_head_greedy_host(None, ctypes.c_void_p(xd.data_ptr()), ctypes.c_void_p(xd.data_ptr()), None, 1e-6,
                                   ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(idx.data_ptr()),
                                   ctypes.c_void_p(host_idx.data_ptr()), 1, 1024, 64, 0, 0,
                                   ctypes.c_void_p(ws.data_ptr()), ws.numel(), None)
    assert st == 7 and b"host memory" in L.mcv_last_error()


@pytest.mark.parametrize("M", [1, 3])
def test_lm_head_w8a8_matches_reference_scan(cuda, M):
    """W8A8 lm_head: the embedding quantized per row on the GPU (layout 2 =
    the oracle's per-channel quantization of its transpose, bit for bit),
    then the fused kernel's index equals the reference's scan - fp16 logits
    RN((acc*ws)*xs), subnormals read as zero, strict '>' first max."""
    import mcv_b200 as mcv
    torch = cuda
    K, V = 1024, 24000
    r = np.random.default_rng(30 + M)
    emb = (r.standard_normal((V, K)) * 0.02).astype(np.float16)
    x = r.standard_normal((M, K)).astype(np.float16)
    ed = torch.from_numpy(emb).cuda()
    wq = torch.empty((V, K), dtype=torch.int8, device="cuda")
    ws = torch.empty(V, dtype=torch.float16, device="cuda")
    mcv.quantize_dense_weight_w8a8(ed, wq, ws, w_layout=2)
    torch.cuda.synchronize()
    wq_ref, ws_ref = oracle.quantize_dense_weight_w8a8(emb.T.copy())
    assert np.array_equal(wq.cpu().numpy(), np.ascontiguousarray(wq_ref.T))
    assert np.array_equal(ws.cpu().numpy().view(np.uint16), np.asarray(ws_ref).view(np.uint16).reshape(-1))

    work = mcv.lm_head_workspace(M)
    idx = torch.empty(M, dtype=torch.int64, device="cuda")
    key = torch.empty(M, dtype=torch.int64, device="cuda")
    for _ in range(2):  # the workspace is left ready for the next call
        mcv.lm_head_argmax_w8a8(torch.from_numpy(x).cuda(), wq, ws, work, out_index=idx, out_key=key)
        torch.cuda.synchronize()
        _, bits = oracle.w8a8_fused(x, wq_ref, ws_ref, nthreads=8)
        bits = np.asarray(bits).reshape(M, V)
        for m in range(M):
            b = bits[m]
            vals = oracle.f16_to_f32(b)
            vals = np.where(((b >> 10) & 0x1F) == 0, np.float32(0.0), vals)  # host h2f: subnormals -> 0
            want = int(np.argmax(vals))  # first maximum = the strict '>' scan (no NaN from int8 dots)
            assert int(idx[m].item()) == want, (m, int(idx[m].item()), want)


def test_lm_head_nan_row_never_wins(cuda):
    """A row whose logit is NaN loses to every number, as in the reference's
    strict '>' scan (language_model.cpp:474-477); the answer equals the
    oracle's over the remaining rows."""
    x, w = synth.lm_head_inputs(1024, 4096, seed=11)
    ref_idx, _, _ = oracle.lm_head_argmax(x, w)
    w = w.copy()
    w[7, 3] = np.float16(np.nan)            # row 7's logit is NaN
    w[int(ref_idx[0]) + 1, 0] = np.float16(np.nan)
    ref2, _, _ = oracle.lm_head_argmax(x, w)
    assert ref2[0] == ref_idx[0]
    idx, _, _ = lm_head(cuda, x, w)
    assert idx[0] == ref_idx[0]
    # all-NaN but one finite row: the finite row wins
    w3 = np.full((64, 1024), np.float16(np.nan), np.float16)
    w3[40] = w[0]
    ref3, _, _ = oracle.lm_head_argmax(x, w3)
    idx3, _, _ = lm_head(cuda, x, w3)
    assert ref3[0] == 40 and idx3[0] == 40


def test_quantize_weight_then_lm_head_w8a8_same_stream(cuda):
    """The weight quantizer followed directly by the W8A8 lm_head on one
    stream, no synchronisation between: the lm_head reads its weights before
    its dependency wait, so the quantizer must not release it early."""
    import mcv_b200 as mcv
    torch = cuda
    K, V = 1024, 65536
    r = np.random.default_rng(77)
    x = r.standard_normal((1, K)).astype(np.float16)
    xd = torch.from_numpy(x).cuda()
    work = mcv.lm_head_workspace(1)
    idx = torch.empty(1, dtype=torch.int64, device="cuda")
    wq = torch.empty((V, K), dtype=torch.int8, device="cuda")
    wsc = torch.empty(V, dtype=torch.float16, device="cuda")
    for trial in range(3):
        emb = (r.standard_normal((V, K)) * 0.02).astype(np.float16)
        ed = torch.from_numpy(emb).cuda()
        wq.fill_(0)
        wsc.fill_(0)
        torch.cuda.synchronize()
        mcv.quantize_dense_weight_w8a8(ed, wq, wsc, w_layout=2)
        mcv.lm_head_argmax_w8a8(xd, wq, wsc, work, out_index=idx)
        torch.cuda.synchronize()
        wq_ref, ws_ref = oracle.quantize_dense_weight_w8a8(emb.T.copy())
        _, bits = oracle.w8a8_fused(x, wq_ref, ws_ref, nthreads=8)
        b = np.asarray(bits).reshape(V)
        vals = np.where(((b >> 10) & 0x1F) == 0, np.float32(0.0), oracle.f16_to_f32(b))
        assert int(idx.item()) == int(np.argmax(vals)), trial
