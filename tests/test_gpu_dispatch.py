"""matmul_decode_dispatch (src/csrc/lib/decoder_layer.cpp:226-244) on the
GPU: for each policy, row count and set of weight formats, the dispatcher's
output equals - bit for bit - the output of the kernel it should have chosen,
called directly."""
import numpy as np
import pytest
import torch

import mcv_b200 as mcv
from mcv_b200 import synth

pytestmark = pytest.mark.gpu

K, N = 1024, 1024


@pytest.fixture(scope="module")
def formats(cuda):
    _, q, z, s = synth.w4a16_inputs(1, K, N, seed=11)
    w4 = mcv.pack_w4a16(q, z, s)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(5)
    dense = (torch.randn((N, K), device="cuda", generator=gen) * 0.02).half()  # [N][K]
    _, w8_kn, w8s = synth.w8a8_inputs(1, K, N, seed=3)
    w8 = torch.from_numpy(np.ascontiguousarray(w8_kn.T)).cuda()  # [N][K]
    w8_scale = torch.from_numpy(w8s).cuda()
    yield dense, w4, w8, w8_scale
    mcv.set_w8a8_decode_mode(None)


def run(x, d):
    out = torch.full((x.shape[0], N), float("nan"), dtype=torch.float16, device="cuda")
    mcv.matmul_decode_dispatch(x, d, out)
    torch.cuda.synchronize()
    return out


def direct(fn, M):
    out = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    fn(out)
    torch.cuda.synchronize()
    return out


def xs(M, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn((M, K), device="cuda", generator=g).half()


def test_w8a8_when_policy_on_and_one_row(formats):
    dense, w4, w8, w8s = formats
    mcv.set_w8a8_decode_mode("all")
    x = xs(1, 1)
    got = run(x, mcv.DecodeWeights.of(dense=dense, w4=w4, w8=w8, w8_scale=w8s))
    want = direct(lambda o: mcv.w8a8_fused(x, w8, w8s, o, w_layout=0), 1)
    assert torch.equal(got, want)


def test_w4a16_when_policy_off(formats):
    dense, w4, w8, w8s = formats
    mcv.set_w8a8_decode_mode("0")
    x = xs(1, 2)
    got = run(x, mcv.DecodeWeights.of(dense=dense, w4=w4, w8=w8, w8_scale=w8s))
    want = direct(lambda o: mcv.matmul_w4a16(x, w4, o), 1)
    assert torch.equal(got, want)


def test_dense_for_several_rows(formats):
    dense, w4, w8, w8s = formats
    mcv.set_w8a8_decode_mode("all")  # W8A8 and W4A16 take one row only
    x = xs(3, 3)
    got = run(x, mcv.DecodeWeights.of(dense=dense, w4=w4, w8=w8, w8_scale=w8s))
    want = direct(lambda o: mcv.matmul_b_transposed(x, dense, o), 3)
    assert torch.equal(got, want)


@pytest.mark.parametrize("M", [2, 8, 40, 80])
def test_int4_without_dense_weight(formats, M):
    """The int4 GEMV up to 32 rows (64 with K <= 4096), the tensor-core GEMM
    beyond."""
    _, w4, _, _ = formats
    mcv.set_w8a8_decode_mode("0")
    x = xs(M, 4 + M)
    got = run(x, mcv.DecodeWeights.of(w4=w4))
    if M <= 32 or (M <= 64 and w4.K <= 4096):
        want = direct(lambda o: mcv.matmul_w4a16(x, w4, o), M)
    else:
        want = direct(lambda o: mcv.matmul_w4a16_gemm(x, w4, o), M)
    assert torch.equal(got, want)


def test_no_usable_format_is_an_error(formats):
    mcv.set_w8a8_decode_mode("0")
    with pytest.raises(mcv.McvError):
        run(xs(1, 9), mcv.DecodeWeights.of())
