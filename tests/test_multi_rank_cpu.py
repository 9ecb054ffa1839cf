"""Host logic of the vocab-sharded lm_head on CPU ranks (gloo, world size 2):
contiguous shards of ceil(V/g) rows with global offsets, order-preserving
64-bit keys combined by a max all-reduce, and failure detection when a rank
dies before the exchange (the survivor's collective ends with an error, no
hang).  No GPU is involved."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _signed(key: int) -> int:
    # flip the top bit so signed int64 order equals unsigned key order
    k = key ^ (1 << 63)
    return k - (1 << 64) if k >= (1 << 63) else k


def _worker(rank, world, port, mode, q):
    import sys
    import torch
    import torch.distributed as dist
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    sys.path[:0] = [os.path.join(root, "oracle"), os.path.join(root, "minicpm-v-4.6-orangepi_b200")]
    import oracle
    from mcv_b200 import synth
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        x, w = synth.lm_head_inputs(64, 10007, seed=3, M=2)
        V = w.shape[0]
        per = (V + world - 1) // world
        a, b = rank * per, min(V, (rank + 1) * per)
        idx, best, _ = oracle.lm_head_argmax(x, np.ascontiguousarray(w[a:b]), n_offset=a)
        keys = torch.tensor([_signed(oracle.argmax_key(float(best[m]), int(idx[m]))) for m in range(2)],
                            dtype=torch.int64)
        if mode == "fail" and rank == 1:
            raise RuntimeError("injected failure before the exchange")
        dist.all_reduce(keys, op=dist.ReduceOp.MAX)
        got = [0xFFFFFFFF - ((int(k) ^ (1 << 63)) & 0xFFFFFFFF) for k in keys]
        ref, _, _ = oracle.lm_head_argmax(x, w)
        q.put((rank, "ok", got, [int(r) for r in ref]))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        q.put((rank, "error", type(e).__name__, str(e)[:200]))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(2):
        r = q.get(timeout=120)
        out[r[0]] = r[1:]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


def test_sharded_keys_combine_to_global_argmax():
    out = _run("ok")
    for rank in (0, 1):
        status, got, ref = out[rank]
        assert status == "ok"
        assert got == ref


def test_rank_failure_is_detected_not_hung():
    out = _run("fail")
    assert out[1][0] == "error" and "injected" in out[1][2]
    assert out[0][0] == "error"  # the survivor's all-reduce fails within the group timeout
