"""Row-parallel reduction over NVLink peer memory (one process per GPU).

A row-parallel FP8 linear (attention-out and FFN-down of the tensor-parallel block
stack) leaves each rank an fp32 partial product P_r = x_r . W_r^T * sx * sw of the full
[M, N] output, to be summed over the ranks.  ``PeerRowReduce`` replaces the GEMM +
NCCL all-reduce with three launches of the qik library per call:

1. ``qik_fp8_gemm_scatter``: the GEMM, whose epilogue stores every finished tile of
   P_r straight into the receive slot of the rank that owns those rows (rows
   [o R, (o + 1) R) belong to rank o, R a multiple of 256), in peer memory, while the
   GEMM goes on with its next tiles; each tile is counted at its owner.
2. ``qik_tp_reduce_gather``: the owner waits for all ranks' tiles of its rows, sums
   them in rank order, adds the bias once, and stores the bf16 rows into every rank's
   output (peer memory again), counting its CTAs there.
3. ``qik_tp_wait``: the rank waits for every owner's rows.

Each rank allocates one workspace tensor (receive slots for two call parities, the
bf16 output for two call parities, the counters), exports it with CUDA IPC and maps
its peers' (``torch.distributed.all_gather_object`` carries the handles).  Counters
only grow: call e waits for e x the per-call count, modulo 2^32, so nothing is reset
between calls.  The receive slot and the output alternate with the parity of the call,
which with the stream order on every rank makes each write land after the previous
reader of that memory is done (see qik_tp.cu).  The output of a call stays valid until
the second-next call of the same ``PeerRowReduce``.

Every wait in the kernels is bounded and reports a timeout in the status word.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib as L

ROW_ALIGN = 256   # rows per owner are a multiple of the GEMM's tallest tile
_ALIGN = 256      # byte alignment of the workspace regions
_MASK32 = 0xFFFFFFFF


class PeerMappingUnavailable(RuntimeError):
    """Raised on every rank when some rank could not map its peers' workspaces (no
    CUDA IPC / peer access between the GPUs); the decision is collective, so all ranks
    take the same fallback."""


def rows_per_owner(M: int, world: int) -> int:
    """Rows each rank owns: ceil(M / world) rounded up to a multiple of 256."""
    per = -(-M // world)
    return -(-per // ROW_ALIGN) * ROW_ALIGN


def _up(n: int) -> int:
    return -(-n // _ALIGN) * _ALIGN


def workspace_layout(M: int, N: int, world: int) -> dict:
    """Byte offsets of the regions of one rank's workspace (identical on every rank):
    recv[parity][src][R][N] fp32, out[parity][M][N] bf16, scatter counters [world]
    (index = source rank), gather counters [world] (index = owner)."""
    R = rows_per_owner(M, world)
    recv = 0
    recv_bytes = 2 * world * R * N * 4
    out = _up(recv + recv_bytes)
    out_bytes = 2 * M * N * 2
    cnt = _up(out + out_bytes)
    gcnt = cnt + _up(world * 4)
    total = gcnt + _up(world * 4)
    return {"R": R, "recv": recv, "slot_bytes": R * N * 4, "out": out, "out_bytes": M * N * 2,
            "cnt": cnt, "gcnt": gcnt, "total": total}


def counter_target(calls: int, per_call: int) -> int:
    """Counter value that completes call number ``calls`` (1-based), modulo 2^32."""
    return (calls * per_call) & _MASK32


class PeerRowReduce:
    """Fused GEMM + sum over ranks for row-parallel FP8 linears with an [M, N] output.

    Collective constructor (every rank of ``group``, same M, N): allocates and maps the
    workspaces.  ``__call__(xq, sx, weight, weight_scale, bias)`` returns the bf16
    [M, N] sum over the ranks (+ bias), a view of the workspace."""

    def __init__(self, M: int, N: int, group=None, device: torch.device | None = None, ctas: int = 128):
        if not (dist.is_available() and dist.is_initialized()):
            raise RuntimeError("PeerRowReduce needs an initialized process group")
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if not 1 <= self.world <= L.TP_MAX_WORLD:
            raise ValueError(f"PeerRowReduce: world {self.world} outside 1..{L.TP_MAX_WORLD}")
        if N % 16:
            raise ValueError("PeerRowReduce: N must be a multiple of 16")
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.M, self.N, self.ctas = M, N, ctas
        self.lay = workspace_layout(M, N, self.world)
        self.lib = L.load()
        self.buf = torch.empty(self.lay["total"], dtype=torch.uint8, device=self.device)
        self.buf[self.lay["cnt"]:].zero_()
        torch.cuda.synchronize(self.device)
        # exchange the workspaces' IPC handles and map the peers'
        hb = self.lib.qik_ipc_handle_bytes()
        handle = ctypes.create_string_buffer(hb)
        off = ctypes.c_uint64(0)
        L.check(self.lib.qik_ipc_export(self.buf.data_ptr(), handle, ctypes.byref(off)), "qik_ipc_export")
        mine = (bytes(handle.raw), int(off.value))
        every: list = [None] * self.world
        dist.all_gather_object(every, mine, group=group)
        self._opened: list[int] = []
        self.base: list[int] = []
        err = ""
        with torch.cuda.device(self.device):
            for p, (h, o) in enumerate(every):
                if p == self.rank:
                    self.base.append(self.buf.data_ptr())
                    continue
                b = ctypes.c_void_p()
                rc = self.lib.qik_ipc_open(ctypes.create_string_buffer(h, hb), ctypes.byref(b))
                if rc != L.QIK_OK:
                    msg = self.lib.qik_last_error()
                    err = f"rank {self.rank} cannot map rank {p}: {msg.decode() if msg else rc}"
                    break
                self._opened.append(b.value)
                self.base.append(b.value + o)
        # every rank learns whether all mappings exist before any kernel writes to a peer
        ok = torch.tensor([0 if err else 1], dtype=torch.int32, device=self.device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        if int(ok.item()) == 0:
            self.close()
            raise PeerMappingUnavailable(err or "a peer rank could not map the workspaces")
        dist.barrier(group=group)
        self.calls = 0
        self.signals = self.lib.qik_fp8_gemm_scatter_signals(M, N, self.lay["R"], self.rank)
        self.status = L.status_word(self.device)
        W = self.world
        self._ptr_arrays = {}
        for parity in (0, 1):
            dst = (ctypes.c_void_p * W)(*[
                self.base[o] + self.lay["recv"] + (parity * W + self.rank) * self.lay["slot_bytes"] for o in range(W)])
            cnt = (ctypes.c_void_p * W)(*[self.base[o] + self.lay["cnt"] + 4 * self.rank for o in range(W)])
            out = (ctypes.c_void_p * W)(*[
                self.base[p] + self.lay["out"] + parity * self.lay["out_bytes"] for p in range(W)])
            gcnt = (ctypes.c_void_p * W)(*[self.base[p] + self.lay["gcnt"] + 4 * self.rank for p in range(W)])
            self._ptr_arrays[parity] = (dst, cnt, out, gcnt)

    def output(self, parity: int) -> torch.Tensor:
        o = self.lay["out"] + parity * self.lay["out_bytes"]
        return self.buf[o:o + self.lay["out_bytes"]].view(torch.bfloat16).view(self.M, self.N)

    def __call__(self, xq: torch.Tensor, sx: torch.Tensor, weight: torch.Tensor, weight_scale: torch.Tensor,
                 bias: torch.Tensor | None = None) -> torch.Tensor:
        M, K = xq.shape
        if M != self.M or weight.shape[0] != self.N or weight.shape[1] != K:
            raise ValueError(f"PeerRowReduce: shapes {tuple(xq.shape)} x {tuple(weight.shape)} do not match "
                             f"[{self.M}, *] x [{self.N}, *]")
        if xq.dtype != torch.float8_e4m3fn or weight.dtype != torch.float8_e4m3fn:
            raise TypeError("PeerRowReduce: e4m3 operands only")
        xq = xq.contiguous()
        self.calls += 1
        parity = self.calls & 1
        dst, cnt, out, gcnt = self._ptr_arrays[parity]
        W, R = self.world, self.lay["R"]
        b = None if bias is None else bias.to(device=self.device, dtype=torch.bfloat16).contiguous()
        stream = L.stream_ptr(self.device)
        with torch.cuda.device(self.device):
            L.check(self.lib.qik_fp8_gemm_scatter(xq.data_ptr(), weight.data_ptr(), M, self.N, K, xq.stride(0),
                                                  weight.stride(0), sx.data_ptr(), weight_scale.data_ptr(), W, R,
                                                  dst, cnt, self.status.data_ptr(), stream), "qik_fp8_gemm_scatter")
            recv = self.base[self.rank] + self.lay["recv"] + parity * W * self.lay["slot_bytes"]
            L.check(self.lib.qik_tp_reduce_gather(recv, self.base[self.rank] + self.lay["cnt"],
                                                  counter_target(self.calls, self.signals), W, self.rank, M, self.N,
                                                  R, L.ptr(b), out, gcnt, self.ctas, self.status.data_ptr(), stream),
                    "qik_tp_reduce_gather")
            L.check(self.lib.qik_tp_wait(self.base[self.rank] + self.lay["gcnt"], counter_target(self.calls, self.ctas),
                                         W, self.status.data_ptr(), stream), "qik_tp_wait")
        return self.output(parity)

    def close(self) -> None:
        """Unmaps the peers' workspaces (after this rank's work on them finished)."""
        if self._opened:
            torch.cuda.synchronize(self.device)
            for b in self._opened:
                self.lib.qik_ipc_close(b)
            self._opened = []

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
