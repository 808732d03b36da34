"""Host logic of the row-sharded projection (multi-GPU), on CPU: shard ranges, zero-row padding
of the last shard, and that gathering every rank's shard-major result through a real
all-gather (gloo, 2 and 3 ranks) and unsharding gives the single-device [M][F] layout.  The
ranks' local GEMM is the oracle's exact dequantization times X (the CUDA GEMM and the unshard
kernel are covered by tests/test_gpu_sharded.py)."""
import os
import socket

import numpy as np
import pytest

from helpers import make_q4_0


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def unshard_np(g, world, m, fs, f):
    """Mirror of unshard_rows_kernel: Y[t][r*fs + j] = G[r][t][j] for j < rows of shard r."""
    y = np.empty((m, f), g.dtype)
    for r in range(world):
        n = min(fs, f - r * fs)
        y[:, r * fs:r * fs + n] = g[r, :, :n]
    return y


def test_shard_rows_ranges():
    from sulimo_b200.sharded import shard_rows
    fs, rng = shard_rows(128256, 8)          # the Llama-3B lm_head of the sharded sweep
    assert fs == 16032 and rng[-1] == (7 * 16032, 128256)
    fs, rng = shard_rows(8192, 3)
    assert fs == 2736 and rng == [(0, 2736), (2736, 5472), (5472, 8192)]
    for f, w in [(8960, 2), (8960, 7), (1536, 8), (200, 2), (8, 1)]:
        fs, rng = shard_rows(f, w)
        assert fs % 8 == 0
        assert rng[0][0] == 0 and rng[-1][1] == f
        assert all(a[1] == b[0] for a, b in zip(rng, rng[1:]))
        assert all(r1 > r0 for r0, r1 in rng)
    with pytest.raises(ValueError):
        shard_rows(16, 4)                     # fs = 8: the 3rd and 4th shard would be empty


def test_shard_weight_pads_last_shard_with_zero_rows():
    import torch
    from sulimo_b200.sharded import shard_weight
    f, k = 200, 64
    ws, wq = make_q4_0(f, k, seed=3)
    st, qt = torch.from_numpy(ws.view(np.int16)), torch.from_numpy(wq)
    s0, q0, fs = shard_weight(st, qt, f, k, 0, 2)
    s1, q1, _ = shard_weight(st, qt, f, k, 1, 2)
    nb = k // 32
    assert fs == 104 and s0.numel() == s1.numel() == fs * nb and q1.numel() == fs * nb * 16
    assert np.array_equal(s0.numpy().view(np.uint16), ws[:fs * nb])
    assert np.array_equal(s1.numpy().view(np.uint16)[:96 * nb], ws[fs * nb:])
    assert not s1.numpy()[96 * nb:].any() and not q1.numpy()[96 * nb * 16:].any()


def _rank(rank, world, port, f, k, m, q):
    import torch
    import torch.distributed as dist
    import oracle.ffi as O
    from sulimo_b200.sharded import shard_weight
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ws, wq = make_q4_0(f, k, seed=11)
        x = np.random.default_rng(12).standard_normal((m, k)).astype(np.float32)
        s_r, q_r, fs = shard_weight(torch.from_numpy(ws.view(np.int16)), torch.from_numpy(wq),
                                    f, k, rank, world)
        w_r = O.dequantize_q4_0_soa(s_r.numpy().view(np.uint16), q_r.numpy(),
                                    fs * k // 32).reshape(fs, k)
        slot = torch.from_numpy((x.astype(np.float64) @ w_r.T.astype(np.float64)).ravel())
        parts = [torch.empty_like(slot) for _ in range(world)]
        dist.all_gather(parts, slot)
        g = torch.cat(parts).numpy().reshape(world, m, fs)
        y = unshard_np(g, world, m, fs, f)
        w = O.dequantize_q4_0_soa(ws, wq, f * k // 32).reshape(f, k)
        full = x.astype(np.float64) @ w.T.astype(np.float64)
        q.put((rank, float(np.abs(y - full).max()), float(np.abs(full).max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,f", [(2, 200), (3, 8192)])
def test_gathered_shards_unshard_to_single_device_layout(world, f):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, f, 64, 5, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, scale in res:
        assert err <= 1e-12 * max(scale, 1.0), (rank, err)
