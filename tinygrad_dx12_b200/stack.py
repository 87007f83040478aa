"""Tensor-parallel packed projection stacks (benchmark configurations c4 and c5).

The reference's packed path ends at one matmul (tinygrad-dx12
``src/tinygrad_dx12/codegen/linalg.py:136-223``); its multi-layer benchmark configurations
chain the projections of a decoder layer over packed weights. One layer here:

    x   = rmsnorm(h)
    qkv = x @ [Wq; Wk; Wv]^T      column-parallel: each rank holds its rows of q, k and v
    h  += allreduce(q @ Wo^T)     row-parallel: each rank holds the K columns of Wo that match
                                  its q rows; partials and the all-reduce are fp32
    x   = rmsnorm(h)
    gu  = x @ [Wg; Wu]^T          column-parallel
    m   = gu[:, :I] * gu[:, I:]   fp32 product rounded to the activation dtype
    h  += allreduce(m @ Wd^T)     row-parallel, fp32

There is no attention: k and v are computed and dropped (their weights stream like a real
layer's). ``rmsnorm(h) = h * rsqrt(mean(h^2) + 1e-6)`` in fp32 keeps the synthetic activations
bounded over 32 or 80 layers. Projections run through ``b200_packed_linear`` (fp32
accumulation); the elementwise steps through ``b200_add_rmsnorm`` / ``b200_gate_mul``; the
all-reduce through ``torch.distributed`` (NCCL between GPUs). Shards are cut from the full
matrices on the device: rows for column-parallel weights, K columns for row-parallel ones
(a K shard must start on a byte and scale-block boundary).
"""

from __future__ import annotations

import dataclasses
import math

import torch

from . import _lib
from . import dtypes as D
from .packed import FORMATS, PackedTensor, stream_ptr

EPS = 1e-6
FLAG_PDL = 0x100  # B200_FLAG_PDL: the decode kernels (M <= 64) may start streaming weights while the previous kernel ends


@dataclasses.dataclass(frozen=True)
class StackConfig:
    hidden: int
    q_dim: int        # q heads x head_dim
    kv_dim: int       # kv heads x head_dim (each of k and v)
    inter: int        # MLP intermediate size
    layers: int
    fmt: str
    block: int        # scale block along K
    scale: str        # "f16u" (fp16 ~U(0.005, 0.02)) or "e8m0" (2^e, e uniform in [-8, -2])
    act: torch.dtype  # activation / output dtype

    def proj_shapes(self) -> dict:
        """(N, K) of every projection of one layer."""
        h, q, kv, i = self.hidden, self.q_dim, self.kv_dim, self.inter
        return {"q": (q, h), "k": (kv, h), "v": (kv, h), "o": (h, q), "gate": (i, h), "up": (i, h), "down": (h, i)}

    def layer_weight_bytes(self) -> int:
        bits = FORMATS[self.fmt][0]
        sb = 1 if self.scale == "e8m0" else 2
        return sum(n * k * bits // 8 + n * (-(-k // self.block)) * sb for n, k in self.proj_shapes().values())


# Benchmark configurations: 8B-shaped INT4 (32 q heads / 8 kv heads of 128) and 70B-shaped FP4
# (64 q heads / 8 kv heads of 128).
C4 = StackConfig(hidden=4096, q_dim=4096, kv_dim=1024, inter=14336, layers=32, fmt="int4", block=128, scale="f16u",
                 act=torch.float16)
C5 = StackConfig(hidden=8192, q_dim=8192, kv_dim=1024, inter=28672, layers=80, fmt="fp4_e2m1", block=32,
                 scale="e8m0", act=torch.bfloat16)


def make_matrix(cfg: StackConfig, layer: int, proj: str, device, seed: int = 0) -> PackedTensor:
    """The full packed matrix of one projection, seeded by (seed, layer, proj) so every rank
    and every world size sees identical weights. Codes are uniform bytes (uniform over the
    format's payloads)."""
    n, k = cfg.proj_shapes()[proj]
    bits = FORMATS[cfg.fmt][0]
    g = torch.Generator(device=device)
    g.manual_seed((seed * 1_000_003 + layer * 101 + list(cfg.proj_shapes()).index(proj)) & 0x7FFFFFFF)
    data = torch.randint(0, 256, (n * k * bits // 8,), dtype=torch.uint8, device=device, generator=g)
    nblk = -(-k // cfg.block)
    if cfg.scale == "e8m0":
        e = torch.randint(-8, -1, (n, nblk), device=device, generator=g)
        scales = (e + 127).to(torch.uint8).view(torch.float8_e8m0fnu)
    else:
        scales = (torch.rand((n, nblk), device=device, generator=g) * 0.015 + 0.005).to(torch.float16)
    return PackedTensor(data, cfg.fmt, (n, k), scales, cfg.block)


# ---- sharding of packed matrices (device-side slicing of the reference byte layout) -------
def shard_rows(w: PackedTensor, start: int, stop: int) -> PackedTensor:
    """Rows [start, stop) of a packed (N, K) matrix (contiguous bytes of the row-major stream)."""
    n, k = w.shape
    bits = FORMATS[w.format][0]
    if (k * bits) % 8:
        raise ValueError("row shards need byte-aligned rows (K * bits % 8 == 0)")
    rb = k * bits // 8
    data = w.data[start * rb:stop * rb].clone()
    scales = w.scales[start:stop].clone() if w.scales is not None else None
    return PackedTensor(data, w.format, (stop - start, k), scales, w.block_size)


def shard_cols(w: PackedTensor, start: int, stop: int) -> PackedTensor:
    """K columns [start, stop) of a packed (N, K) matrix. The shard must start on a byte
    boundary of every row and on a scale-block boundary."""
    n, k = w.shape
    bits = FORMATS[w.format][0]
    if (start * bits) % 8 or (stop * bits) % 8 or (k * bits) % 8:
        raise ValueError("column shards must start and end on byte boundaries")
    if w.scales is not None and (start % w.block_size or (stop % w.block_size and stop != k)):
        raise ValueError("column shards must align with scale blocks")
    rb = k * bits // 8
    data = w.data[:n * rb].view(n, rb)[:, start * bits // 8:stop * bits // 8].contiguous().view(-1)
    scales = None
    if w.scales is not None:
        scales = w.scales[:, start // w.block_size:-(-stop // w.block_size)].contiguous()
    return PackedTensor(data, w.format, (n, stop - start), scales, w.block_size)


def concat_rows(ws: list[PackedTensor]) -> PackedTensor:
    """Stack packed matrices with equal K along N (one fused projection call)."""
    k = ws[0].shape[1]
    assert all(w.shape[1] == k and w.format == ws[0].format and w.block_size == ws[0].block_size for w in ws)
    data = torch.cat([w.data for w in ws])
    scales = torch.cat([w.scales for w in ws]) if ws[0].scales is not None else None
    return PackedTensor(data, ws[0].format, (sum(w.shape[0] for w in ws), k), scales, ws[0].block_size)


def split(total: int, world: int, rank: int, align: int = 1) -> tuple[int, int]:
    """Even split of `total` over `world` ranks; every boundary a multiple of `align`."""
    if total % (world * align):
        raise ValueError(f"{total} does not split over {world} ranks in multiples of {align}")
    part = total // world
    return rank * part, (rank + 1) * part


@dataclasses.dataclass
class LayerShard:
    qkv: PackedTensor   # [q_r; k_r; v_r] rows
    o: PackedTensor     # Wo columns matching q_r
    gu: PackedTensor    # [gate_r; up_r] rows
    down: PackedTensor  # Wd columns matching gate_r / up_r
    q_rows: int         # q rows of this rank (the width of q_r)
    inter_rows: int     # gate rows of this rank


def shard_layer(full: dict, cfg: StackConfig, rank: int, world: int) -> LayerShard:
    """This rank's tensor-parallel shard of one layer's full matrices."""
    kalign = max(cfg.block, 8)  # K shards of o / down on scale-block and byte boundaries
    q0, q1 = split(cfg.q_dim, world, rank, 1)
    kv0, kv1 = split(cfg.kv_dim, world, rank, 1)
    i0, i1 = split(cfg.inter, world, rank, 1)
    if q0 % kalign or i0 % kalign or (q1 - q0) % kalign or (i1 - i0) % kalign:
        raise ValueError("row-parallel K shards must be multiples of the scale block")
    qkv = concat_rows([shard_rows(full["q"], q0, q1), shard_rows(full["k"], kv0, kv1), shard_rows(full["v"], kv0, kv1)])
    gu = concat_rows([shard_rows(full["gate"], i0, i1), shard_rows(full["up"], i0, i1)])
    return LayerShard(qkv=qkv, o=shard_cols(full["o"], q0, q1), gu=gu, down=shard_cols(full["down"], i0, i1),
                      q_rows=q1 - q0, inter_rows=i1 - i0)


# ---- compute back-ends ----------------------------------------------------------------------
class CudaOps:
    """The B200 library: fused packed projections and the glue kernels."""

    def __init__(self, group=None):
        self.group = group

    def linear(self, w: PackedTensor, x: torch.Tensor, out_dtype: torch.dtype) -> torch.Tensor:
        from .linalg import _packed_linear

        return _packed_linear(w, x, out_dtype, "auto", FLAG_PDL if x.shape[0] <= 64 else 0)

    def add_rmsnorm(self, h: torch.Tensor, partial: torch.Tensor | None, x_out: torch.Tensor | None) -> None:
        _lib.call("b200_add_rmsnorm", h.data_ptr(), _lib.DT[D.name(h.dtype)],
                  partial.data_ptr() if partial is not None else None,
                  x_out.data_ptr() if x_out is not None else None,
                  _lib.DT[D.name(x_out.dtype)] if x_out is not None else 0, h.shape[0], h.shape[1], EPS,
                  stream_ptr(h.device))

    def gate_mul(self, gu: torch.Tensor, out: torch.Tensor) -> None:
        _lib.call("b200_gate_mul", gu.data_ptr(), _lib.DT[D.name(gu.dtype)], out.data_ptr(), _lib.DT[D.name(out.dtype)],
                  gu.shape[0], out.shape[1], stream_ptr(gu.device))

    def all_reduce(self, t: torch.Tensor) -> None:
        import torch.distributed as dist

        if dist.is_initialized() and dist.get_world_size(self.group) > 1:
            dist.all_reduce(t, group=self.group)

    def row_reduce(self, w: PackedTensor, inp: torch.Tensor, h: torch.Tensor, x: torch.Tensor, slot: int) -> None:
        """h += allreduce(inp @ w^T) (fp32 partials); x = rmsnorm(h)."""
        p = self.linear(w, inp, torch.float32)
        self.all_reduce(p)
        self.add_rmsnorm(h, p, x)


class PeerReducer:
    """Partial buffers shared by all ranks through CUDA IPC, and the fused one-shot reduction.

    Each rank owns one device allocation: fp32 partial slots [2][world][rows_max][hidden] (slot
    [b][q] holds rank q's partial of reduction parity b), the flag words every rank writes
    ([world][rows_max]) and this rank's epoch counters. The allocation's IPC handle is exchanged
    over the process group and every rank maps every peer's. A rank's row-parallel projection
    pushes its partial into slot [b][rank] of every rank (the GEMV epilogue stores to all of
    them); the reduction then reads only local memory.
    """

    def __init__(self, rows_max: int, hidden: int, group=None, timeout_s: float = 5.0):
        import ctypes

        import torch.distributed as dist

        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("peer reduction supports up to 8 ranks")
        self.rows_max, self.hidden, self.group = rows_max, hidden, group
        self.timeout_ns = int(timeout_s * 1e9)
        self.dev = torch.cuda.current_device()
        self.part_bytes = rows_max * hidden * 4
        slots = 2 * self.world * self.part_bytes
        flag_bytes = self.world * rows_max * 4
        total = slots + flag_bytes + rows_max * 4
        base = ctypes.c_void_p()
        _lib.call("b200_malloc", self.dev, total, ctypes.byref(base))
        self.base = base.value
        zeros = torch.zeros(total, dtype=torch.uint8, device=f"cuda:{self.dev}")
        _lib.call("b200_memcpy", self.base, zeros.data_ptr(), total, 2, None)
        torch.cuda.synchronize()
        handle = ctypes.create_string_buffer(64)
        _lib.call("b200_ipc_get_handle", self.base, handle)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        self.bases, self.opened = [], []
        for q, hq in enumerate(handles):
            if q == self.rank:
                self.bases.append(self.base)
                continue
            p = ctypes.c_void_p()
            _lib.call("b200_ipc_open", ctypes.create_string_buffer(hq, 64), ctypes.byref(p))
            self.bases.append(p.value)
            self.opened.append(p.value)
        P = ctypes.c_void_p * 8
        w = self.world

        def slot(base, b, src):
            return base + (b * w + src) * self.part_bytes

        order = [self.rank] + [q for q in range(w) if q != self.rank]  # local destination first
        self._push = [(ctypes.c_void_p * w)(*[slot(self.bases[q], b, self.rank) for q in order]) for b in (0, 1)]
        self._partials = [P(*[slot(self.base, b, q) for q in range(w)]) for b in (0, 1)]
        self._flags = P(*[b_ + slots for b_ in self.bases])
        self.epoch = self.base + slots + flag_bytes
        dist.barrier(group=group)  # every rank's flags are zero before anyone signals

    def push_targets(self, slot: int):
        """Where this rank's partial of reduction parity `slot` goes: its slot in every rank."""
        return self._push[slot]

    def reduce(self, slot: int, h: torch.Tensor, x: torch.Tensor | None) -> None:
        m, hidden = h.shape
        if m > self.rows_max or hidden != self.hidden:
            raise ValueError("peer reduction: rows or width beyond the shared buffers")
        _lib.call("b200_peer_allreduce_add_rmsnorm", self._partials[slot], self._flags, self.epoch, self.rank,
                  self.world, self.rows_max, self.timeout_ns, h.data_ptr(), _lib.DT[D.name(h.dtype)],
                  x.data_ptr() if x is not None else None, _lib.DT[D.name(x.dtype)] if x is not None else 0, m, hidden,
                  EPS, stream_ptr(h.device))

    def close(self) -> None:
        for p in self.opened:
            _lib.call("b200_ipc_close", p)
        self.opened = []
        if self.base:
            _lib.call("b200_free", self.dev, self.base)
            self.base = 0


class PeerOps(CudaOps):
    """CudaOps whose row-parallel projections push fp32 partials straight into every rank's
    shared buffer and reduce them with the fused kernel (rows <= rows_max)."""

    def __init__(self, rows_max: int, hidden: int, group=None):
        super().__init__(group)
        self.reducer = PeerReducer(rows_max, hidden, group)

    def row_reduce(self, w: PackedTensor, inp: torch.Tensor, h: torch.Tensor, x: torch.Tensor, slot: int) -> None:
        from .linalg import _packed_linear_multi

        if h.shape[0] > self.reducer.rows_max:  # beyond the shared buffers: NCCL all-reduce
            return super().row_reduce(w, inp, h, x, slot)
        _packed_linear_multi(w, inp, self.reducer.push_targets(slot), torch.float32, h.shape[1],
                             FLAG_PDL if inp.shape[0] <= 64 else 0)
        self.reducer.reduce(slot, h, x)

    def close(self) -> None:
        self.reducer.close()


class TPStack:
    """One rank's shard of a packed projection stack and its forward pass."""

    def __init__(self, cfg: StackConfig, rank: int = 0, world: int = 1, device="cuda", layers: int | None = None,
                 seed: int = 0, ops=None, matrix_fn=None):
        self.cfg, self.rank, self.world = cfg, rank, world
        self.ops = ops or CudaOps()
        self.nlayers = cfg.layers if layers is None else layers
        mk = matrix_fn or (lambda layer, proj: make_matrix(cfg, layer, proj, device, seed))
        self.layers = []
        for layer in range(self.nlayers):
            full = {p: mk(layer, p) for p in cfg.proj_shapes()}
            self.layers.append(shard_layer(full, cfg, rank, world))
            del full

    def weight_bytes(self) -> int:
        """Packed bytes + scale bytes this rank streams per forward pass."""
        tot = 0
        for L in self.layers:
            for w in (L.qkv, L.o, L.gu, L.down):
                tot += w.data.numel() + (w.scales.numel() * w.scales.element_size() if w.scales is not None else 0)
        return tot

    def forward(self, h: torch.Tensor) -> torch.Tensor:
        """h: (M, hidden) in the activation dtype, replicated on every rank; updated in place."""
        cfg, ops = self.cfg, self.ops
        m = h.shape[0]
        x = torch.empty_like(h)
        mbuf = torch.empty((m, self.layers[0].inter_rows if self.layers else 0), dtype=cfg.act, device=h.device)
        ops.add_rmsnorm(h, None, x)
        if self.world == 1:  # unsharded: nothing to reduce whatever the process group holds
            row_reduce = lambda w, inp, hh, xx, slot: _local_row_reduce(ops, w, inp, hh, xx)  # noqa: E731
        else:
            row_reduce = getattr(ops, "row_reduce", None) or (
                lambda w, inp, hh, xx, slot: _generic_row_reduce(ops, w, inp, hh, xx))
        for L in self.layers:
            qkv = ops.linear(L.qkv, x, cfg.act)
            row_reduce(L.o, qkv[:, :L.q_rows], h, x, 0)
            gu = ops.linear(L.gu, x, cfg.act)
            ops.gate_mul(gu, mbuf)
            row_reduce(L.down, mbuf, h, x, 1)
        return h


def _local_row_reduce(ops, w, inp, h, x) -> None:
    ops.add_rmsnorm(h, ops.linear(w, inp, torch.float32), x)


def _generic_row_reduce(ops, w, inp, h, x) -> None:
    p = ops.linear(w, inp, torch.float32)
    ops.all_reduce(p)
    ops.add_rmsnorm(h, p, x)
