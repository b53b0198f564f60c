"""Multi-GPU execution of the FP8 DiT hot path: one process per GPU, torch.distributed.

Three layouts (the reference itself is single-GPU; these serve the token-row sweep and the
tensor-parallel layer stack):

* **Shards** -- token rows (or the two CFG branches) are independent work: each rank
  runs the unchanged single-GPU path on its own rows, with no collective on the data
  path.  A per-tensor dynamic scale is a reduction over the whole tensor, so
  ``quantize_sharded(..., global_amax=True)`` adds one 4-byte all-reduce(MAX) of the
  amax bits; every shard is then quantized exactly as the 1-GPU run quantizes the
  full tensor (fp32 bit patterns of |x| order like integers, so an int32 MAX is the
  bits of the global amax).  Without it each shard is quantized like an independent
  call of the reference (what the reference does per CFG branch).

* **Tensor parallel block stack** -- weights are quantized once on the full tensor
  and their e4m3 bytes are sharded, so every rank holds exactly the 1-GPU weights and
  scale.  QKV (fused, 3 x heads) and FFN-up are column-parallel (QKV by heads, so
  attention runs on local heads with no communication); attention-out and FFN-down
  are row-parallel: their input scale needs the global amax (4-byte all-reduce MAX),
  their fp32 partial products are summed with an NCCL all-reduce, and the bias is
  added once after the sum.

* **Sequence parallel** (``TPBlock(sequence_parallel=True)``) -- the same stack with the
  activations between the linears kept as row shards: a row-parallel linear's fp32
  partial products are reduce-scattered (each rank receives the sum of its own rows),
  the bias add and bf16 cast run on those rows only, and a column-parallel linear
  quantizes its local rows with the global scale (4-byte all-reduce MAX) and
  all-gathers the e4m3 bytes (1 byte per element) before its GEMM.  Per row-parallel
  linear a rank then moves (world-1)/world of the fp32 product once (reduce-scatter)
  plus (world-1)/world of the e4m3 activation, instead of an fp32 all-reduce (twice
  the product) followed by a replicated amax and pack of the whole activation; the
  e4m3 bytes equal the 1-GPU quantization of the whole tensor.

The arithmetic goes through an ``ops`` object: ``QikOps`` (the CUDA kernels, the
default and the only product path) or a test double with the same methods.
"""
from __future__ import annotations

import warnings

import torch
import torch.distributed as dist
import torch.nn as nn

from . import _lib as L


class QikOps:
    """The qik CUDA kernels behind the operations the parallel layer composes."""

    def amax_bits(self, x: torch.Tensor) -> torch.Tensor:
        from .fp8 import amax_bits
        return amax_bits(x)

    def pack(self, x: torch.Tensor, amax: torch.Tensor):
        from .fp8 import quantize_from_amax
        return quantize_from_amax(x, amax)

    def gemm(self, xq, sx, wq, sw, bias=None, out_dtype=torch.bfloat16, epilogue=L.EPI_SCALE, amax_out=None,
             out=None):
        from .fp8 import fp8_gemm
        return fp8_gemm(xq, sx, wq, sw, bias=bias, out_dtype=out_dtype, epilogue=epilogue, amax_out=amax_out,
                        out=out)

    def zeros_amax(self, device) -> torch.Tensor:
        return torch.zeros(1, dtype=torch.int32, device=device)

    def attention(self, q, k, v, L):
        from .triton_attention import block_causal_flash_attention
        return block_causal_flash_attention(q, k, v, L, None)

    def bias_bf16(self, x: torch.Tensor, bias: torch.Tensor | None, amax: torch.Tensor) -> torch.Tensor:
        """bf16(x + bias) of fp32 rows, max|out| accumulated into ``amax``."""
        xc = x.contiguous()
        out = torch.empty(xc.shape, dtype=torch.bfloat16, device=x.device)
        b = None if bias is None else bias.contiguous()
        lib = L.load()
        with torch.cuda.device(x.device):
            L.check(lib.qik_rows_bias_bf16(xc.data_ptr(), xc.shape[0], xc.shape[1], L.ptr(b), out.data_ptr(),
                                           amax.data_ptr(), L.stream_ptr()), "qik_rows_bias_bf16")
        return out


_comm_streams: dict[int, torch.cuda.Stream] = {}


def _comm_stream(device: torch.device) -> torch.cuda.Stream:
    """One side stream per device for collectives that overlap compute."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    st = _comm_streams.get(idx)
    if st is None:
        st = torch.cuda.Stream(device=torch.device("cuda", idx))
        _comm_streams[idx] = st
    return st


def _world(group) -> tuple[int, int]:
    if not dist.is_available() or not dist.is_initialized():
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


def row_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous balanced split of n rows: the first n % world ranks get one more."""
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def allreduce_amax_(amax: torch.Tensor, group=None) -> torch.Tensor:
    """In place: integer MAX of the amax bit patterns over the group."""
    if _world(group)[1] > 1:
        dist.all_reduce(amax, op=dist.ReduceOp.MAX, group=group)
    return amax


def _nccl(group) -> bool:
    return dist.get_backend(group) == "nccl"


def reduce_scatter_rows(part: torch.Tensor, group=None) -> torch.Tensor:
    """This rank's rows [M / world, N] of the sum over the ranks of ``part`` [M, N]
    (M a multiple of world): NCCL's reduce-scatter; gloo, which has none, sums with an
    all-reduce and keeps the rank's rows."""
    rank, world = _world(group)
    if world == 1:
        return part
    M = part.shape[0]
    if M % world:
        raise ValueError(f"reduce_scatter_rows: {M} rows do not split evenly over {world} ranks")
    if _nccl(group):
        out = torch.empty((M // world,) + tuple(part.shape[1:]), dtype=part.dtype, device=part.device)
        dist.reduce_scatter_tensor(out, part.contiguous(), op=dist.ReduceOp.SUM, group=group)
        return out
    full = part.contiguous().clone()
    dist.all_reduce(full, op=dist.ReduceOp.SUM, group=group)
    return full[rank * (M // world):(rank + 1) * (M // world)].contiguous()


def all_gather_rows(local: torch.Tensor, group=None) -> torch.Tensor:
    """The ranks' equal row shards concatenated in rank order (e4m3 moved as bytes)."""
    _, world = _world(group)
    if world == 1:
        return local
    fp8 = local.dtype == torch.float8_e4m3fn
    src = (local.view(torch.uint8) if fp8 else local).contiguous()
    if _nccl(group):
        full = torch.empty((world * src.shape[0],) + tuple(src.shape[1:]), dtype=src.dtype, device=src.device)
        dist.all_gather_into_tensor(full, src, group=group)
    else:
        parts = [torch.empty_like(src) for _ in range(world)]
        dist.all_gather(parts, src, group=group)
        full = torch.cat(parts, 0)
    return full.view(torch.float8_e4m3fn) if fp8 else full


def quantize_sharded(x_local: torch.Tensor, group=None, global_amax: bool = True, ops=None):
    """Dynamic per-tensor e4m3 quantization of this rank's rows.  With global_amax the
    scale is the one of the full (concatenated) tensor."""
    ops = ops or QikOps()
    amax = ops.amax_bits(x_local)
    if global_amax:
        allreduce_amax_(amax, group)
    return ops.pack(x_local, amax)


# ------------------------------------------------------------------ weight sharding
def shard_rows(w: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Output-feature (row) shard of a [N, K] weight for a column-parallel linear."""
    n = w.shape[0]
    if n % world:
        raise ValueError(f"{n} output features do not split over {world} ranks")
    step = n // world
    return w[rank * step:(rank + 1) * step].contiguous()


def shard_cols(w: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Input-feature (column) shard of a [N, K] weight for a row-parallel linear."""
    k = w.shape[1]
    if k % world:
        raise ValueError(f"{k} input features do not split over {world} ranks")
    step = k // world
    return w[:, rank * step:(rank + 1) * step].contiguous()


def shard_qkv_heads(w: torch.Tensor, heads: int, head_dim: int, rank: int, world: int) -> torch.Tensor:
    """Rows of the fused QKV weight ([q; k; v], each heads * head_dim rows, the layout of
    quantize_offline.py:80) that produce this rank's heads, as [q_l; k_l; v_l]."""
    if heads % world:
        raise ValueError(f"{heads} heads do not split over {world} ranks")
    hl = heads // world
    inner = heads * head_dim
    if w.shape[0] != 3 * inner:
        raise ValueError("fused QKV weight must have 3 * heads * head_dim rows")
    raw = w.view(torch.uint8) if w.dtype == torch.float8_e4m3fn else w
    parts = [raw[p * inner + rank * hl * head_dim: p * inner + (rank + 1) * hl * head_dim] for p in range(3)]
    out = torch.cat(parts, 0).contiguous()
    return out.view(w.dtype) if w.dtype == torch.float8_e4m3fn else out


def shard_vector(b: torch.Tensor | None, rank: int, world: int) -> torch.Tensor | None:
    if b is None:
        return None
    step = b.shape[0] // world
    return b[rank * step:(rank + 1) * step].contiguous()


def shard_qkv_bias(b: torch.Tensor | None, heads: int, head_dim: int, rank: int, world: int):
    if b is None:
        return None
    return shard_qkv_heads(b[:, None], heads, head_dim, rank, world)[:, 0].contiguous()


# ------------------------------------------------------------------ layers
class ColumnParallelFP8Linear(nn.Module):
    """y_local = x . W_local^T (+ b_local): this rank's output features.  The input is
    the full activation, replicated on every rank, so every rank computes the same
    dynamic scale without communicating."""

    def __init__(self, weight: torch.Tensor, weight_scale: torch.Tensor, bias: torch.Tensor | None, ops=None):
        super().__init__()
        self.register_buffer("weight", weight)
        self.register_buffer("weight_scale", weight_scale)
        if bias is not None:
            self.register_buffer("bias", bias)
        else:
            self.bias = None
        self.ops = ops or QikOps()

    @classmethod
    def from_full(cls, weight, weight_scale, bias, rank, world, qkv_heads: tuple[int, int] | None = None, ops=None):
        if qkv_heads is not None:
            w = shard_qkv_heads(weight, qkv_heads[0], qkv_heads[1], rank, world)
            b = shard_qkv_bias(bias, qkv_heads[0], qkv_heads[1], rank, world)
        else:
            w, b = shard_rows(weight, rank, world), shard_vector(bias, rank, world)
        return cls(w, weight_scale.clone(), b, ops)

    def forward(self, x: torch.Tensor, epilogue: int = L.EPI_SCALE, amax_out: torch.Tensor | None = None):
        x2 = x.reshape(-1, x.shape[-1])
        amax = self.ops.amax_bits(x2)
        xq, sx = self.ops.pack(x2, amax)
        return self.ops.gemm(xq, sx, self.weight, self.weight_scale, self.bias, epilogue=epilogue, amax_out=amax_out)

    def forward_gathered(self, x_local: torch.Tensor, amax: torch.Tensor | None = None, group=None,
                         epilogue: int = L.EPI_SCALE, amax_out: torch.Tensor | None = None):
        """Sequence parallel: the input is this rank's rows.  They are quantized with the
        scale of the whole input (``amax``: max|x_local| if a producer accumulated it,
        made global by a 4-byte all-reduce MAX), the e4m3 rows of all ranks gathered,
        and the GEMM runs over every row for this rank's output features."""
        x2 = x_local.reshape(-1, x_local.shape[-1])
        if amax is None:
            amax = self.ops.amax_bits(x2)
        allreduce_amax_(amax, group)
        xq_local, sx = self.ops.pack(x2, amax)
        xq = all_gather_rows(xq_local, group)
        return self.ops.gemm(xq, sx, self.weight, self.weight_scale, self.bias, epilogue=epilogue, amax_out=amax_out)


class RowParallelFP8Linear(nn.Module):
    """y = sum_ranks x_local . W_local^T (+ b): the input holds this rank's slice of the
    input features.  The dynamic scale is global (4-byte all-reduce MAX of the amax
    bits), the fp32 partial products are summed with an all-reduce, and the bias is
    added once after the sum.

    With ``chunks`` > 1 on GPUs (more than one rank) the GEMM runs in row blocks: the
    all-reduce of block i runs on a side stream while the GEMM of block i + 1 runs.
    Every rank issues the same collectives in the same order; the sum is the same as
    one all-reduce of the whole partial product (the reduction is per element).  The
    default is one block: measured on 2 B200 the overlapped form was slower (the
    NCCL kernels occupy SMs the persistent GEMM grid counts on).

    With ``comm="peer"`` (GPUs, more than one rank) the sum runs over NVLink peer
    memory instead (``qik.tp_comm.PeerRowReduce``): the GEMM's epilogue stores each
    finished fp32 tile into the receive slot of the rank owning those rows while the
    GEMM goes on, the owner sums its rows in rank order, adds the bias and stores bf16
    rows into every rank's output.  Its workspace is set up collectively at the first
    call with a given row count; the output stays valid until this module's
    second-next call.  ``comm="auto"`` (the default) takes the peer-memory sum for two
    ranks and the NCCL all-reduce for more: measured on B200 for the 4-block TP stack,
    4.29 ms (peer) against 4.99 ms (NCCL) on 2 GPUs, but 5.19 ms against 4.53 ms on 4,
    where each rank ships three quarters of its fp32 partial product and NCCL reduces in
    the NVSwitch."""

    def __init__(self, weight: torch.Tensor, weight_scale: torch.Tensor, bias: torch.Tensor | None, group=None,
                 ops=None, chunks: int = 1, comm: str = "auto"):
        super().__init__()
        if comm not in ("auto", "nccl", "peer"):
            raise ValueError(f"RowParallelFP8Linear: comm must be 'auto', 'nccl' or 'peer', not {comm!r}")
        self.comm = comm
        self._peer: dict = {}
        self.chunks = chunks
        self.register_buffer("weight", weight)
        self.register_buffer("weight_scale", weight_scale)
        if bias is not None:
            self.register_buffer("bias", bias)
        else:
            self.bias = None
        self.group = group
        self.ops = ops or QikOps()

    @classmethod
    def from_full(cls, weight, weight_scale, bias, rank, world, group=None, ops=None, chunks: int = 1,
                  comm: str = "auto"):
        return cls(shard_cols(weight, rank, world), weight_scale.clone(), bias, group, ops, chunks, comm)

    def forward_quantized(self, xq: torch.Tensor, sx: torch.Tensor) -> torch.Tensor:
        world = _world(self.group)[1]
        M = xq.shape[0]
        peer = self.comm == "peer" or (self.comm == "auto" and world == 2)
        if world > 1 and xq.is_cuda and peer and self.chunks == 1:
            red = self._peer.get(M)
            if red is None:
                from .tp_comm import PeerMappingUnavailable, PeerRowReduce
                try:
                    red = PeerRowReduce(M, self.weight.shape[0], self.group, xq.device)
                except PeerMappingUnavailable as e:
                    # collective decision: every rank falls back to the all-reduce
                    warnings.warn(f"RowParallelFP8Linear: peer-memory reduction unavailable ({e}); "
                                  "using the NCCL all-reduce")
                    red = False
                self._peer[M] = red
            if red is not False:
                return red(xq, sx, self.weight, self.weight_scale, self.bias)
        if world > 1 and xq.is_cuda and self.chunks > 1 and M >= 2 * self.chunks:
            part = self._gemm_allreduce_overlapped(xq, sx)
        else:
            part = self.ops.gemm(xq, sx, self.weight, self.weight_scale, None, out_dtype=torch.float32)
            if world > 1:
                dist.all_reduce(part, op=dist.ReduceOp.SUM, group=self.group)
        if self.bias is not None:
            part = part + self.bias.float()
        return part.to(torch.bfloat16)

    def _gemm_allreduce_overlapped(self, xq: torch.Tensor, sx: torch.Tensor) -> torch.Tensor:
        M = xq.shape[0]
        N = self.weight.shape[0]
        part = torch.empty(M, N, dtype=torch.float32, device=xq.device)
        cur = torch.cuda.current_stream(xq.device)
        comm = _comm_stream(xq.device)
        for c in range(self.chunks):
            lo, hi = row_range(M, c, self.chunks)
            blk = part[lo:hi]
            self.ops.gemm(xq[lo:hi], sx, self.weight, self.weight_scale, None, out_dtype=torch.float32, out=blk)
            done = torch.cuda.Event()
            done.record(cur)
            comm.wait_event(done)
            with torch.cuda.stream(comm):
                dist.all_reduce(blk, op=dist.ReduceOp.SUM, group=self.group)
        cur.wait_stream(comm)
        part.record_stream(comm)
        return part

    def forward(self, x_local: torch.Tensor, amax: torch.Tensor | None = None) -> torch.Tensor:
        x2 = x_local.reshape(-1, x_local.shape[-1])
        if amax is None:
            amax = self.ops.amax_bits(x2)
        allreduce_amax_(amax, self.group)
        xq, sx = self.ops.pack(x2, amax)
        return self.forward_quantized(xq, sx)

    def forward_scattered(self, xq: torch.Tensor, sx: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Sequence parallel: the sum over the ranks of the partial products, reduce-
        scattered by rows (M a multiple of the world size), so this rank receives its
        own rows only; the bias is added to them once and their max|.| accumulated for
        the next FP8 linear.  Returns (bf16 rows [M / world, N], amax bits)."""
        part = self.ops.gemm(xq, sx, self.weight, self.weight_scale, None, out_dtype=torch.float32)
        rows = reduce_scatter_rows(part, self.group)
        amax = self.ops.zeros_amax(xq.device)
        return self.ops.bias_bf16(rows, self.bias, amax), amax


def tp_ffn(x: torch.Tensor, up: ColumnParallelFP8Linear, down: RowParallelFP8Linear) -> torch.Tensor:
    """down(gelu_tanh(up(x))) with up column-parallel and down row-parallel: the GELU
    epilogue of the local up-projection accumulates the local amax of the hidden
    activation, which one 4-byte all-reduce makes global before the pack."""
    ops = up.ops
    amax = ops.zeros_amax(x.device)
    h = up(x, epilogue=L.EPI_GELU_TANH, amax_out=amax)
    allreduce_amax_(amax, down.group)
    hq, sh = ops.pack(h, amax)
    return down.forward_quantized(hq, sh)


def tp_ffn_sp(h_local: torch.Tensor, h_amax: torch.Tensor | None, up: ColumnParallelFP8Linear,
              down: RowParallelFP8Linear) -> tuple[torch.Tensor, torch.Tensor]:
    """Sequence-parallel tp_ffn: this rank's rows in (with their max|.| when known), this
    rank's rows of down(gelu_tanh(up(h))) out, with their max|.|."""
    ops = up.ops
    amax = ops.zeros_amax(h_local.device)
    hid = up.forward_gathered(h_local, h_amax, down.group, epilogue=L.EPI_GELU_TANH, amax_out=amax)
    allreduce_amax_(amax, down.group)
    hq, sh = ops.pack(hid, amax)
    return down.forward_scattered(hq, sh)


class TPBlock(nn.Module):
    """The linears + attention of one DiT block, tensor parallel over heads / hidden
    features: QKV (column, by heads) -> block-causal attention on the local heads ->
    attention-out (row) -> FFN up (column, GELU-tanh) -> FFN down (row).

    With ``sequence_parallel`` the block's input and output are this rank's token rows
    (rows [rank * M / world, (rank + 1) * M / world); M a multiple of the world size):
    the column-parallel linears gather the e4m3 rows of every rank, the row-parallel
    ones reduce-scatter their partial products (``forward_gathered``,
    ``forward_scattered``); the NCCL (or gloo) collectives carry both."""

    def __init__(self, qkv, out, up, down, heads_local: int, head_dim: int, sequence_parallel: bool = False):
        super().__init__()
        self.qkv, self.out, self.up, self.down = qkv, out, up, down
        self.hl, self.d = heads_local, head_dim
        self.sequence_parallel = sequence_parallel

    @classmethod
    def from_full(cls, full: dict, heads: int, head_dim: int, rank: int, world: int, group=None, ops=None,
                  chunks: int = 1, comm: str = "auto", sequence_parallel: bool = False):
        """full: name -> (weight e4m3 [N, K], weight_scale [1], bias or None) for
        'qkv', 'out', 'up', 'down' (unsharded, quantized once).  ``chunks``: row blocks of
        the row-parallel GEMMs whose all-reduce overlaps the next block's GEMM;
        ``comm``: "peer" (reduction over NVLink peer memory fused with the GEMM,
        RowParallelFP8Linear), "nccl" (all-reduce) or "auto" (the default: "peer" for two
        ranks, "nccl" for more)."""
        qkv = ColumnParallelFP8Linear.from_full(*full["qkv"], rank, world, qkv_heads=(heads, head_dim), ops=ops)
        out = RowParallelFP8Linear.from_full(*full["out"], rank, world, group, ops, chunks, comm)
        up = ColumnParallelFP8Linear.from_full(*full["up"], rank, world, ops=ops)
        down = RowParallelFP8Linear.from_full(*full["down"], rank, world, group, ops, chunks, comm)
        return cls(qkv, out, up, down, heads // world, head_dim, sequence_parallel)

    def forward(self, x: torch.Tensor, batch: int, seq: int, prefix_lengths: torch.Tensor,
                x_amax: torch.Tensor | None = None) -> torch.Tensor:
        """x: the whole activation [batch * seq, width] (replicated), or with
        ``sequence_parallel`` this rank's rows of it (``x_amax``: their max|.| when the
        producer accumulated it, e.g. the previous block's ``forward_sp``)."""
        if self.sequence_parallel:
            return self.forward_sp(x, batch, seq, prefix_lengths, x_amax)[0]
        M = x.shape[0]
        qkv = self.qkv(x).view(batch, seq, 3, self.hl, self.d)
        o = self.qkv.ops.attention(qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2], prefix_lengths)
        h = self.out(o.reshape(M, self.hl * self.d))
        return tp_ffn(h, self.up, self.down)

    def forward_sp(self, x_local: torch.Tensor, batch: int, seq: int, prefix_lengths: torch.Tensor,
                   x_amax: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """Sequence parallel: this rank's rows in, this rank's rows out with their
        max|.| (the next block's ``x_amax``)."""
        group = self.out.group
        M = batch * seq
        qkv = self.qkv.forward_gathered(x_local, x_amax, group).view(batch, seq, 3, self.hl, self.d)
        o = self.qkv.ops.attention(qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2], prefix_lengths)
        o2 = o.reshape(M, self.hl * self.d)
        amax = self.qkv.ops.amax_bits(o2)
        allreduce_amax_(amax, group)
        oq, so = self.qkv.ops.pack(o2, amax)
        h_local, h_amax = self.out.forward_scattered(oq, so)
        return tp_ffn_sp(h_local, h_amax, self.up, self.down)
