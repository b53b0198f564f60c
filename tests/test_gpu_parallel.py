"""Multi-GPU parity (NCCL, one process per GPU; needs >= 2 GPUs, skipped otherwise).

* token-row shards quantized with the 4-byte global-amax all-reduce produce exactly
  the bytes and scale of the single-GPU quantization of the whole tensor;
* the tensor-parallel DiT block (QKV by heads, attention on local heads, row-parallel
  out / FFN-down with fp32 partial all-reduce) matches the single-GPU block within
  the BASELINE tolerances, in both forms (one all-reduce, or row blocks whose
  all-reduces run on a side stream);
* the sequence-parallel block (row shards in and out: reduce-scatter of the partial
  products, e4m3 rows all-gathered with the global scale) equals the all-reduce form
  bit for bit on each rank's rows, two blocks in a row;
* with the row-parallel sums over NVLink peer memory (qik.tp_comm.PeerRowReduce:
  GEMM epilogue stores into the owner's memory, owner reduce + bf16 gather) the block
  is bit-identical to the all-reduce form (same fp32 partial products; for two ranks
  the fp32 sum of two terms does not depend on the order), over three successive calls
  (receive slots and counters alternate / grow with the call number), and a direct
  reduction with ragged ownership (M = 1000: owner 1 holds 488 rows) equals the
  partial product + all-reduce + bias of the same operands.
"""
import datetime
import os
import pickle
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import golden_inputs as GI

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _block_weights(dev, heads=24, d=128, k=3072, hidden=12288):
    from qik import fp8 as F
    full = {}
    for i, (name, n, kk) in enumerate([("qkv", 3 * heads * d, k), ("out", k, heads * d), ("up", hidden, k),
                                       ("down", k, hidden)]):
        w = GI.randn_bf16(200 + i, (n, kk), 0.02).to(dev)
        q, s = F.quantize_weight_tensorwise(w)
        b = GI.randn_bf16(210 + i, (n,), 0.1).to(dev) if name in ("qkv", "out") else None
        full[name] = (q, s, b)
    return full


def _worker(rank, world, port, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        from qik import parallel as PX
        res = {}
        x = GI.outlier_activations(5, 4352, 3072)
        x[3, 3] = 900.0
        lo, hi = PX.row_range(x.shape[0], rank, world)
        q, s = PX.quantize_sharded(x[lo:hi].contiguous().to(dev))
        res["q"] = q.view(torch.uint8).cpu().numpy()
        res["s"] = float(s.item())
        B, S, heads, d = 2, 512, 24, 128
        full = _block_weights(dev)
        blk = PX.TPBlock.from_full(full, heads, d, rank, world, comm="nccl")
        xb = GI.randn_bf16(220, (B * S, 3072)).to(dev)
        Lp = torch.arange(S, dtype=torch.int32, device=dev)
        Lp[64:] = S - 1
        res["block"] = blk(xb, B, S, Lp).float().cpu().numpy()
        # sequence parallel: this rank's rows in and out, two blocks in a row
        bsp = PX.TPBlock.from_full(full, heads, d, rank, world, sequence_parallel=True)
        lo_r, hi_r = rank * (B * S // world), (rank + 1) * (B * S // world)
        y1, a1 = bsp.forward_sp(xb[lo_r:hi_r].contiguous(), B, S, Lp)
        y1c = y1.clone()
        y2, _ = bsp.forward_sp(y1, B, S, Lp, a1)
        res["block_sp"] = (lo_r, hi_r, y1c.float().cpu().numpy(), y2.float().cpu().numpy())
        res["block_twice"] = blk(blk(xb, B, S, Lp), B, S, Lp).float().cpu().numpy()
        # row-parallel GEMMs in 4 row blocks, each all-reduce on a side stream
        blk4 = PX.TPBlock.from_full(full, heads, d, rank, world, chunks=4, comm="nccl")
        res["block4"] = blk4(xb, B, S, Lp).float().cpu().numpy()
        # row-parallel sums over peer memory, three calls
        blkp = PX.TPBlock.from_full(full, heads, d, rank, world, comm="peer")
        res["block_peer"] = [blkp(xb, B, S, Lp).float().cpu().numpy() for _ in range(3)]
        # direct reduction, ragged ownership, bias
        from qik import _lib as L
        from qik import fp8 as F
        from qik.tp_comm import PeerRowReduce
        M, N, K = 1000, 512, 256
        a = GI.randn_bf16(230 + rank, (M, K)).to(dev)
        w = GI.randn_bf16(232 + rank, (N, K), 0.05).to(dev)
        bias = GI.randn_bf16(234, (N,), 0.1).to(dev)
        aq, sa = F.quantize_tensorwise(a)
        wq, sw = F.quantize_weight_tensorwise(w)
        red = PeerRowReduce(M, N, device=dev)
        got = [red(aq, sa, wq, sw, bias).clone() for _ in range(3)]
        part = F.fp8_gemm(aq, sa, wq, sw, out_dtype=torch.float32)
        dist.all_reduce(part)
        want = (part + bias.float()).to(torch.bfloat16)
        res["direct_equal"] = [bool(torch.equal(g, want)) for g in got]
        res["status"] = L.device_status(dev)
        torch.cuda.synchronize()
        dist.barrier()
        red.close()
        for lin in (blkp.out, blkp.down):
            for r in lin._peer.values():
                assert r, "peer-memory reduction fell back to NCCL"
                r.close()
        with open(os.path.join(outdir, f"r{rank}.pkl"), "wb") as f:
            pickle.dump(res, f)
    finally:
        dist.destroy_process_group()


def test_sharded_quantization_and_tp_block_on_two_gpus():
    from oracle import oracle as O
    from qik import fp8 as F
    from qik import parallel as PX
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(2, _free_port(), d), nprocs=2, start_method="spawn", join=True)
        res = []
        for r in range(2):
            with open(os.path.join(d, f"r{r}.pkl"), "rb") as f:
                res.append(pickle.load(f))
    # single-GPU references in this process
    dev = torch.device("cuda", 0)
    x = GI.outlier_activations(5, 4352, 3072)
    x[3, 3] = 900.0
    q1, s1 = F.quantize_tensorwise(x.to(dev))
    assert np.array_equal(np.concatenate([r["q"] for r in res], 0), q1.view(torch.uint8).cpu().numpy())
    assert all(r["s"] == float(s1.item()) for r in res)
    B, S, heads, dh = 2, 512, 24, 128
    full = _block_weights(dev)
    blk = PX.TPBlock.from_full(full, heads, dh, 0, 1)
    xb = GI.randn_bf16(220, (B * S, 3072)).to(dev)
    Lp = torch.arange(S, dtype=torch.int32, device=dev)
    Lp[64:] = S - 1
    ref = blk(xb, B, S, Lp).float().cpu()
    for r in res:
        y = torch.from_numpy(r["block"])
        assert O.relf(y, ref) <= 5e-3
        # the blocked form: same partial products, summed block by block (its GEMM
        # blocks may use another tile configuration, so the gate is the tolerance)
        assert O.relf(torch.from_numpy(r["block4"]), ref) <= 5e-3
        assert r["status"] == 0
        assert all(np.array_equal(yp, r["block"]) for yp in r["block_peer"])
        # sequence parallel (reduce-scatter + e4m3 all-gather): on two ranks the same
        # two-term sums and the same e4m3 bytes as the all-reduce form
        lo_r, hi_r, y1, y2 = r["block_sp"]
        assert np.array_equal(y1, r["block"][lo_r:hi_r])
        assert np.array_equal(y2, r["block_twice"][lo_r:hi_r])
        assert r["direct_equal"] == [True, True, True]
