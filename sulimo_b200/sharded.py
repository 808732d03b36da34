"""Row-sharded Q4_0 projection over several GPUs (one process per GPU, torch.distributed/NCCL).

The reference runs on one device.  Its Q4_0 projections shard naturally by output rows: with the
SoA layout (crates/sulimo-core/src/repack.rs:45-81) rows [r0, r1) of a [F][K] tensor are the
contiguous subranges scales[r0*K/32 : r1*K/32] and quants[r0*K/2 : r1*K/2], whole 32-element
K blocks untouched.  Rank r holds `fs` rows (the last rank's tail padded with zero-scale rows,
whose outputs are 0 and dropped), computes Y_r = X W_r^T with the tcgen05 GEMM into its slot of
a shard-major buffer G[world][M][fs], and one NCCL all-gather (the path's only exchange step)
fills G on every rank.  `unshard_rows` then writes the row-major Y[M][F] the single-GPU GEMM
produces (or the caller consumes G shard-major).
"""
import sulimo_b200 as sb

ROW_ALIGN = 8  # the GEMM needs a multiple of 8 output rows


def shard_rows(f, world, align=ROW_ALIGN):
    """Rows per shard (`fs`, a multiple of `align`) and the [r0, r1) range of every rank.

    The last range may be shorter than fs; every range is non-empty."""
    if f <= 0 or world <= 0:
        raise ValueError("rows and world size must be positive")
    fs = -(-f // world)
    fs = -(-fs // align) * align
    if (world - 1) * fs >= f:
        raise ValueError(f"{f} rows cannot give {world} non-empty shards of {fs} rows")
    return fs, [(r * fs, min(f, (r + 1) * fs)) for r in range(world)]


def shard_weight(scales, quants, f, k, rank, world):
    """This rank's rows of a Q4_0 SoA tensor (torch tensors: scales f16 bits, quants bytes),
    padded to exactly fs rows with zero scales.  Returns (scales_r, quants_r, fs)."""
    import torch
    nb = k // 32
    fs, ranges = shard_rows(f, world)
    r0, r1 = ranges[rank]
    sc = scales[r0 * nb:r1 * nb]
    qu = quants[r0 * nb * 16:r1 * nb * 16]
    if r1 - r0 < fs:
        pad = fs - (r1 - r0)
        sc = torch.cat([sc, torch.zeros(pad * nb, dtype=scales.dtype, device=scales.device)])
        qu = torch.cat([qu, torch.zeros(pad * nb * 16, dtype=quants.dtype, device=quants.device)])
    return sc.contiguous(), qu.contiguous(), fs


class ShardedQ4Projection:
    """Y[M][F] = X[M][K] W^T for a W[F][K] Q4_0 tensor split by rows over the process group."""

    def __init__(self, ctx, scales_r, quants_r, f, k, fs, group=None):
        import torch.distributed as dist
        self.ctx, self.scales, self.quants = ctx, scales_r, quants_r
        self.f, self.k, self.fs, self.group = f, k, fs, group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0

    def buffers(self, m, out_dtype=sb.OUT_F16):
        """(gather buffer [world*m*fs], row-major output [m*F]) for m tokens."""
        import torch
        dt = torch.float16 if out_dtype == sb.OUT_F16 else torch.float32
        g = torch.empty(self.world * m * self.fs, dtype=dt, device="cuda")
        y = torch.empty(m * self.f, dtype=dt, device="cuda")
        return g, y

    def local_gemm(self, x, m, gather, out_dtype=sb.OUT_F16):
        """This rank's rows into its slot of the shard-major buffer (no communication)."""
        n = m * self.fs
        slot = gather[self.rank * n:(self.rank + 1) * n]
        sb.gemm_q4_0_f16(self.ctx, self.scales, self.quants, x, slot, self.fs, self.k, m,
                         out_dtype)
        return slot

    def all_gather(self, m, gather):
        """The exchange step: every rank's [m][fs] slot to every rank (in place, NCCL)."""
        import torch.distributed as dist
        if self.world == 1:
            return
        n = m * self.fs
        dist.all_gather_into_tensor(gather, gather[self.rank * n:(self.rank + 1) * n],
                                    group=self.group)

    def forward(self, x, m, gather, y=None, out_dtype=sb.OUT_F16):
        """GEMM + all-gather (+ row-major unshard when `y` is given).  Returns y or gather."""
        self.local_gemm(x, m, gather, out_dtype)
        self.all_gather(m, gather)
        if y is None:
            return gather
        if self.world == 1 and self.fs == self.f:
            y.copy_(gather)
        else:
            sb.unshard_rows(self.ctx, gather, y, self.world, m, self.fs, self.f)
        return y


class FusedShardedQ4Projection(ShardedQ4Projection):
    """The same projection with the all-gather fused into the GEMM: every rank's epilogue
    stores its output tiles straight into every rank's row-major Y[M][F] over NVLink (peer
    mappings of library buffers exchanged as CUDA IPC handles) and bumps every rank's arrival
    counter; `forward` then waits (bounded, on the device) until this rank's counter has all
    ranks' CTAs.  No NCCL on the data path, no unshard pass.  Y and the counters are allocated
    once for up to `m_max` tokens.  Every rank makes the same sequence of calls (the counter
    targets and the release epochs advance by one call each time), so this path is not captured
    in graphs.  Y may be read until the next call: a call stores into a peer's Y only after that
    peer's own next call has started on its stream (the kernel's release handshake), so readers
    of the returned Y that the caller enqueues on this context's stream before its next call
    always see this call's result.
    """

    RELEASE_OFFSET = 128  # bytes from a rank's arrival counter to its release word

    def __init__(self, ctx, scales_r, quants_r, f, k, fs, m_max, out_dtype=sb.OUT_F16,
                 group=None):
        import ctypes as C

        import torch
        import torch.distributed as dist
        from sulimo_b200 import capi
        super().__init__(ctx, scales_r, quants_r, f, k, fs, group)
        if f % 8:
            raise ValueError("F must be a multiple of 8")
        self.m_max, self.out_dtype = m_max, out_dtype
        self.es = 2 if out_dtype == sb.OUT_F16 else 4
        self.y_buf = ctx.alloc(m_max * f * self.es)
        self.flag_buf = ctx.alloc(256)
        ctx.write(self.flag_buf, bytes(256))
        handles = torch.zeros(2, 64, dtype=torch.uint8)
        hbuf = (C.c_uint8 * 64)()
        for i, b in enumerate((self.y_buf, self.flag_buf)):
            capi.call("sulimo_cuda_ipc_handle", b, hbuf)
            handles[i] = torch.tensor(list(hbuf), dtype=torch.uint8)
        if self.world > 1:
            allh = torch.empty(self.world, 2, 64, dtype=torch.uint8, device="cuda")
            dist.all_gather_into_tensor(allh, handles.cuda(), group=group)
            allh = allh.cpu()
        else:
            allh = handles.unsqueeze(0)
        self.opened = []
        bases, flags = [], []
        for r in range(self.world):
            if r == self.rank:
                bases.append(ctx.device_ptr(self.y_buf))
                flags.append(ctx.device_ptr(self.flag_buf))
                continue
            ptrs = []
            for i in range(2):
                out = C.c_void_p()
                h = (C.c_uint8 * 64)(*allh[r, i].tolist())
                capi.call("sulimo_cuda_ipc_open", ctx.handle, h, C.byref(out))
                ptrs.append(out.value)
                self.opened.append(out.value)
            bases.append(ptrs[0])
            flags.append(ptrs[1])
        self.bases = (C.c_void_p * self.world)(*bases)
        self.flags = (C.c_void_p * self.world)(*flags)
        self.own_flag = ctx.device_ptr(self.flag_buf)
        # the release word sits 128 bytes into each rank's flag buffer (its own cache line)
        self.releases = (C.c_void_p * self.world)(*[p + self.RELEASE_OFFSET for p in flags])
        self.epoch_arrivals = 0
        self.calls = 0
        self.valid = min(f - self.rank * fs, fs)

    def forward_fused(self, x, m):
        """Y[m][F] on every rank (device pointer of this rank's copy); x [m][k] f16."""
        import ctypes as C
        from sulimo_b200 import capi
        if m > self.m_max:
            raise ValueError("m exceeds the buffers' m_max")
        tiles = C.c_uint()
        self.calls = (self.calls + 1) & 0xFFFFFFFF or 1
        capi.call("sulimo_cuda_gemm_q4_0_f16_allgather", self.ctx.handle, self.scales.data_ptr(),
                  self.quants.data_ptr(), x.data_ptr(), self.fs, self.valid, self.k, m,
                  self.out_dtype, self.bases, self.f, self.rank * self.fs, self.flags,
                  self.releases, self.world, self.rank, self.calls, C.byref(tiles))
        # every rank launches the same tile count (equal fs), so one call adds world * tiles
        self.epoch_arrivals = (self.epoch_arrivals + self.world * tiles.value) & 0xFFFFFFFF
        capi.call("sulimo_cuda_wait_counter", self.ctx.handle, self.own_flag, self.epoch_arrivals)
        return self.ctx.device_ptr(self.y_buf)

    def read(self, m):
        """Host copy of Y[m][F] (numpy f16 / f32)."""
        import numpy as np
        out = np.empty(m * self.f, np.float16 if self.es == 2 else np.float32)
        self.ctx.read(self.y_buf, out)
        return out.reshape(m, self.f)

    def close(self):
        from sulimo_b200 import capi
        for p in self.opened:
            capi.call("sulimo_cuda_ipc_close", self.ctx.handle, p)
        self.opened = []
        self.ctx.free(self.y_buf)
        self.ctx.free(self.flag_buf)
