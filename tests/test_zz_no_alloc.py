"""The allocation-free lm_head entry point (mcv_lm_head_argmax_noalloc).

Some callers cannot allocate device memory, so they cannot hand
mcv_lm_head_argmax a workspace; this entry point uses a fixed scratch array
inside the library instead.  Here it is called through the C ABI twice in a
row (the array keeps the first call's contents) and must give the same argmax
keys and indices as the workspace entry point on the same inputs.  The file
is named to be collected last.
"""
import ctypes

import numpy as np
import pytest

from mcv_b200 import synth

pytestmark = pytest.mark.gpu


def test_noalloc_matches_workspace_entry_point(cuda):
    import mcv_b200
    torch = cuda
    L = mcv_b200.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call, (M, N, off, fp16) in enumerate([(1, 248094, 0, 0), (3, 40000, 1000, 1)]):
        x, w = synth.lm_head_inputs(1024, N, seed=50 + call, M=M)
        xd = torch.from_numpy(x).cuda()
        wd = torch.from_numpy(w).cuda()
        ws = mcv_b200.lm_head_workspace(M)
        ref_key = torch.empty(M, dtype=torch.int64, device="cuda")
        ref_idx = torch.empty(M, dtype=torch.int64, device="cuda")
        st = L.mcv_lm_head_argmax(xd.data_ptr(), wd.data_ptr(), ref_key.data_ptr(), ref_idx.data_ptr(), M, 1024, N,
                                  off, fp16, ws.data_ptr(), ws.numel(), stream)
        assert st == 0
        key = torch.full((M,), -1, dtype=torch.int64, device="cuda")
        idx = torch.full((M,), -1, dtype=torch.int64, device="cuda")
        st = L.mcv_lm_head_argmax_noalloc(xd.data_ptr(), wd.data_ptr(), key.data_ptr(), idx.data_ptr(), M, 1024, N,
                                          off, fp16, stream)
        assert st == 0, L.mcv_last_error()
        torch.cuda.synchronize()
        # argmax keys and indices are integers: exact match
        assert np.array_equal(key.cpu().numpy(), ref_key.cpu().numpy())
        assert np.array_equal(idx.cpu().numpy(), ref_idx.cpu().numpy())
    assert L.mcv_lm_head_noalloc_max_bytes() >= L.mcv_lm_head_workspace_size(8)
    fake = ctypes.c_void_p(16)
    assert L.mcv_lm_head_argmax_noalloc(fake, fake, fake, fake, 9, 1024, 100, 0, 0, stream) == 2
