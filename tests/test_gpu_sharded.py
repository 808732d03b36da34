"""GPU parity of the row-sharded projection: the unshard kernel (exact copy semantics, 16-byte
and element paths, uneven last shard), the shards' GEMMs reassembled on one GPU against the
single-device GEMM and the oracle, and -- with two or more GPUs -- the NCCL all-gather path
itself (one process per GPU)."""
import os
import socket

import numpy as np
import pytest

import oracle.ffi as O
import sulimo_b200 as sb
from gpu_util import dev, empty, host
from helpers import make_q4_0, rel_l2

pytestmark = pytest.mark.gpu


def unshard_np(g, world, m, fs, f):
    y = np.empty((m, f), g.dtype)
    for r in range(world):
        n = min(fs, f - r * fs)
        y[:, r * fs:r * fs + n] = g[r, :, :n]
    return y


@pytest.mark.parametrize("dtype", [np.float16, np.float32])
@pytest.mark.parametrize("world,m,fs,f", [(3, 7, 24, 72), (3, 7, 24, 70), (1, 5, 40, 40),
                                          (8, 3, 16032, 128256), (2, 1, 104, 200)])
def test_unshard_rows_exact(ctx, dtype, world, m, fs, f):
    import torch
    g = np.random.default_rng(world * 100 + f).standard_normal((world, m, fs)).astype(dtype)
    out = empty(m * f, torch.float16 if dtype == np.float16 else torch.float32)
    sb.unshard_rows(ctx, dev(g.ravel()), out, world, m, fs, f)
    ctx.finish()
    assert np.array_equal(host(out).reshape(m, f), unshard_np(g, world, m, fs, f))


def test_unshard_rows_rejects_bad_shapes(ctx):
    import torch
    t = empty(64, torch.float16)
    with pytest.raises(sb.SulimoError):
        sb.unshard_rows(ctx, t, t, 4, 1, 8, 16)   # (world-1)*fs >= F: an empty shard


def run_gemm(ctx, sc, qu, x, m_feat, k, n, out_dtype=sb.OUT_F32):
    import torch
    out = empty(n * m_feat, torch.float32 if out_dtype == sb.OUT_F32 else torch.float16)
    sb.gemm_q4_0_f16(ctx, sc, qu, x, out, m_feat, k, n, out_dtype)
    return out


@pytest.mark.parametrize("world,f,k,m", [(4, 8192, 3072, 16), (3, 1000, 512, 33), (8, 2048, 256, 1)])
def test_shards_reassembled_on_one_gpu(ctx, world, f, k, m):
    """Each 'rank' computed in turn on cuda:0 into its slot of the shard-major buffer, then the
    unshard kernel: equals the single-device GEMM (rel-L2 2e-3, the GEMM's bar) and the oracle."""
    import torch
    from sulimo_b200.sharded import shard_weight
    ws, wq = make_q4_0(f, k, seed=f + k)
    x = np.random.default_rng(m).standard_normal(m * k).astype(np.float16)
    dws, dwq, dx = dev(ws), dev(wq), dev(x)
    gath = None
    for r in range(world):
        s_r, q_r, fs = shard_weight(dws, dwq, f, k, r, world)
        if gath is None:
            gath = empty(world * m * fs, torch.float32)
        sb.gemm_q4_0_f16(ctx, s_r, q_r, dx, gath[r * m * fs:(r + 1) * m * fs], fs, k, m,
                         sb.OUT_F32)
    y = empty(m * f, torch.float32)
    sb.unshard_rows(ctx, gath, y, world, m, fs, f)
    full = run_gemm(ctx, dws, dwq, dx, f, k, m)
    ctx.finish()
    assert rel_l2(host(y), host(full)) <= 2e-3
    rows = [0, m - 1]
    xs = np.concatenate([x[t * k:(t + 1) * k] for t in rows])
    orc = O.gemm_q4_0_f16_f32out(ws, wq, xs.view(np.uint16), f, k, len(rows), threads=8)
    got = host(y).reshape(m, f)[rows].ravel()
    assert rel_l2(got, orc) <= 2e-3


def _nccl_rank(rank, world, port, f, k, m, q):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from sulimo_b200.sharded import ShardedQ4Projection, shard_weight
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        ctx = sb.CudaContext(rank, stream=torch.cuda.current_stream())
        ws, wq = make_q4_0(f, k, seed=5)
        x = np.random.default_rng(6).standard_normal(m * k).astype(np.float16)
        dws, dwq, dx = dev(ws), dev(wq), dev(x)
        s_r, q_r, fs = shard_weight(dws, dwq, f, k, rank, world)
        proj = ShardedQ4Projection(ctx, s_r, q_r, f, k, fs)
        g, y = proj.buffers(m, sb.OUT_F32)
        proj.forward(dx, m, g, y, sb.OUT_F32)
        full = run_gemm(ctx, dws, dwq, dx, f, k, m)
        ctx.finish()
        q.put((rank, rel_l2(host(y), host(full))))
        ctx.close()
    finally:
        dist.destroy_process_group()


def test_nccl_all_gather_two_gpus():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    c = mp.get_context("spawn")
    q = c.Queue()
    procs = [c.Process(target=_nccl_rank, args=(r, 2, port, 8192, 3072, 16, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, err in res:
        assert err <= 2e-3, (rank, err)


# ---- the all-gather fused into the GEMM epilogue (peer stores over NVLink + counters) ---------

def test_fused_allgather_single_rank(ctx):
    """world 1: the fused epilogue stores into the rank's own Y and the counter wait passes;
    two calls in a row (the counter target advances)."""
    from sulimo_b200.sharded import FusedShardedQ4Projection
    f, k = 1024, 512
    ws, wq = make_q4_0(f, k, seed=31)
    dws, dwq = dev(ws), dev(wq)
    proj = FusedShardedQ4Projection(ctx, dws, dwq, f, k, f, m_max=48, out_dtype=sb.OUT_F32)
    try:
        for m, seed in ((48, 1), (17, 2)):
            x = np.random.default_rng(seed).standard_normal(m * k).astype(np.float16)
            proj.forward_fused(dev(x), m)
            ctx.finish()
            got = proj.read(m)
            ref = O.gemm_q4_0_f16_f32out(ws, wq, x.view(np.uint16), f, k, m, threads=8)
            assert rel_l2(got.ravel(), ref) <= 2e-3
    finally:
        proj.close()


def _fused_rank(rank, world, port, f, k, m, q):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from sulimo_b200 import capi
    from sulimo_b200.sharded import FusedShardedQ4Projection, shard_weight
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        ctx = sb.CudaContext(rank, stream=torch.cuda.current_stream())
        ws, wq = make_q4_0(f, k, seed=8)
        dws, dwq = dev(ws), dev(wq)
        s_r, q_r, fs = shard_weight(dws, dwq, f, k, rank, world)
        proj = FusedShardedQ4Projection(ctx, s_r, q_r, f, k, fs, m_max=m, out_dtype=sb.OUT_F32)
        # calls back to back with no host synchronisation: each result is read by a copy kernel
        # enqueued on this rank's stream before its next call, while the peer's next call may
        # already be running; the release handshake keeps the peer from overwriting Y early
        xs = [dev(np.random.default_rng(seed).standard_normal(m * k).astype(np.float16))
              for seed in SEEDS]
        snaps = [torch.empty(m * f, dtype=torch.float32, device="cuda") for _ in SEEDS]
        for x, snap in zip(xs, snaps):
            y = proj.forward_fused(x, m)
            capi.call("sulimo_cuda_unshard_rows", ctx.handle, y, snap.data_ptr(), 1, m, f, f, 4)
        ctx.finish()
        outs = [host(t).reshape(m, f) for t in snaps]
        dist.barrier()  # no rank closes its mappings while a peer may still store into them
        proj.close()
        q.put((rank, outs))
        ctx.close()
    finally:
        dist.destroy_process_group()


SEEDS = (9, 10, 11, 12, 13, 14)


def test_fused_allgather_two_gpus():
    """Both ranks end with the same full Y for each of six back-to-back calls, equal to the
    single-device projection of that call's input."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    f, k, m = 2000, 1024, 40   # uneven shards: 1000 rows each; ragged token tile
    c = mp.get_context("spawn")
    q = c.Queue()
    procs = [c.Process(target=_fused_rank, args=(r, 2, port, f, k, m, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    ws, wq = make_q4_0(f, k, seed=8)
    for i, seed in enumerate(SEEDS):
        assert np.array_equal(res[0][i].view(np.uint32), res[1][i].view(np.uint32))
        x = np.random.default_rng(seed).standard_normal(m * k).astype(np.float16)
        ref = O.gemm_q4_0_f16_f32out(ws, wq, x.view(np.uint16), f, k, m, threads=8)
        assert rel_l2(res[0][i].ravel(), ref) <= 2e-3
