"""Sharded lm_head across GPUs: the NCCL all-reduce path and the fused
peer-mailbox path against the CPU oracle (argmax indices exact), including
replay inside a CUDA graph, plus the bounded wait of the fused path when a
peer never arrives (one GPU, one spinning kernel, error reported)."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _paths():
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    return [os.path.join(root, "oracle"), os.path.join(root, "minicpm-v-4.6-orangepi_b200")]


def _rank_main(rank, world, port, q):
    import sys
    sys.path[:0] = _paths()
    import torch
    import torch.distributed as dist
    import mcv_b200 as mcv
    from mcv_b200 import synth
    try:
        torch.cuda.set_device(rank)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        M, K, V = 2, 1024, 248094
        x, w = synth.lm_head_inputs(K, V, seed=8, M=M)
        per = (V + world - 1) // world
        a, b = rank * per, min(V, (rank + 1) * per)
        xd = torch.from_numpy(x).cuda()
        wd = torch.from_numpy(np.ascontiguousarray(w[a:b])).cuda()
        ws = mcv.lm_head_workspace(M)
        key = torch.empty(M, dtype=torch.int64, device="cuda")
        idx = torch.empty(M, dtype=torch.int64, device="cuda")
        results = {}
        # NCCL path
        uid = [mcv.NcclComm.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, 0)
        comm = mcv.NcclComm(world, rank, uid[0])
        mcv.lm_head_argmax_allreduce(comm, xd, wd, ws, key, idx, n_offset=a)
        torch.cuda.synchronize()
        results["nccl"] = idx.cpu().tolist()
        comm.destroy()
        # fused peer-mailbox path, 3 eager calls then 2 graph replays
        ctx = mcv.P2PContext(world, rank)
        hs = [None] * world
        dist.all_gather_object(hs, ctx.ipc_handle)
        ctx.connect(hs)
        dist.barrier()
        seen = []
        for _ in range(3):
            idx.fill_(-7)
            mcv.lm_head_argmax_p2p(ctx, xd, wd, ws, key, idx, n_offset=a)
            torch.cuda.synchronize()
            seen.append(idx.cpu().tolist())
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        with torch.cuda.graph(g, stream=s):
            mcv.lm_head_argmax_p2p(ctx, xd, wd, ws, key, idx, n_offset=a)
        dist.barrier()
        for _ in range(2):
            idx.fill_(-7)
            g.replay()
            torch.cuda.synchronize()
            seen.append(idx.cpu().tolist())
        # one-call host path on the same context (pinned x in, index written
        # straight into pinned host memory)
        x_host = torch.from_numpy(x).pin_memory()
        x_dev = torch.empty_like(xd)
        idx_host = torch.full((M,), -7, dtype=torch.int64).pin_memory()
        for _ in range(2):
            idx_host.fill_(-7)
            mcv.lm_head_greedy_host(x_host, x_dev, wd, idx, idx_host, ws, ctx=ctx, n_offset=a)
            seen.append(idx_host.tolist())
        results["p2p"] = seen
        results["p2p_errors"] = ctx.errors()
        dist.barrier()
        ctx.destroy()
        if rank == 0:
            import oracle
            ref, _, gap = oracle.lm_head_argmax(x, w, nthreads=8)
            results["ref"] = [int(r) for r in ref]
            results["gap"] = [float(v) for v in gap]
        q.put((rank, "ok", results))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", repr(e)[:400]))


def test_sharded_lm_head_two_gpus(cuda):
    torch = cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(2):
        r = q.get(timeout=600)
        out[r[0]] = r[1:]
    for p in procs:
        p.join(timeout=120)
    for rank in (0, 1):
        assert out[rank][0] == "ok", out[rank]
    ref = out[0][1]["ref"]
    assert min(out[0][1]["gap"]) > 1e-4
    for rank in (0, 1):
        res = out[rank][1]
        assert res["nccl"] == ref
        for got in res["p2p"]:
            assert got == ref
        assert res["p2p_errors"] == 0


def _idle_peer(port_q, done_q):
    import sys
    sys.path[:0] = _paths()
    import torch
    import mcv_b200 as mcv
    torch.cuda.set_device(0)
    ctx = mcv.P2PContext(2, 1)
    port_q.put(ctx.ipc_handle)
    done_q.get(timeout=300)  # never calls the kernel: its key never arrives
    ctx.destroy()


def test_p2p_missing_peer_times_out(cuda):
    """Rank 1 creates its mailbox but never runs the kernel; rank 0's kernel
    gives up after its 1 s bound, records the error and returns index -1."""
    torch = cuda
    import mcv_b200 as mcv
    mpc = mp.get_context("spawn")
    hq, dq = mpc.Queue(), mpc.Queue()
    p = mpc.Process(target=_idle_peer, args=(hq, dq))
    p.start()
    try:
        h1 = hq.get(timeout=300)
        ctx = mcv.P2PContext(2, 0)
        ctx.connect([ctx.ipc_handle, h1])
        x = torch.randn((1, 256), device="cuda").half()
        w = torch.randn((1000, 256), device="cuda").half()
        ws = mcv.lm_head_workspace(1)
        key = torch.empty(1, dtype=torch.int64, device="cuda")
        idx = torch.empty(1, dtype=torch.int64, device="cuda")
        mcv.lm_head_argmax_p2p(ctx, x, w, ws, key, idx, n_offset=0)
        torch.cuda.synchronize()
        assert idx.item() == -1
        assert ctx.errors() & 1
        assert ctx.errors() == 0  # cleared by the read
        # indices travel in 24 bits of a mailbox word: larger ones are refused
        # on the host, before any launch
        with pytest.raises(mcv.McvError):
            mcv.lm_head_argmax_p2p(ctx, x, w, ws, key, idx, n_offset=(1 << 24) - 1000)
        ctx.destroy()
    finally:
        dq.put("done")
        p.join(timeout=60)
