"""Multi-GPU parity (NCCL, one process per GPU; needs >= 2 GPUs, skipped otherwise).

* token-row shards quantized with the 4-byte global-amax all-reduce produce exactly
  the bytes and scale of the single-GPU quantization of the whole tensor;
* the tensor-parallel DiT block (QKV by heads, attention on local heads, row-parallel
  out / FFN-down with fp32 partial all-reduce) matches the single-GPU block within
  the BASELINE tolerances, in both forms (one all-reduce, or row blocks whose
  all-reduces run on a side stream).
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
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
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
        blk = PX.TPBlock.from_full(full, heads, d, rank, world)
        xb = GI.randn_bf16(220, (B * S, 3072)).to(dev)
        Lp = torch.arange(S, dtype=torch.int32, device=dev)
        Lp[64:] = S - 1
        res["block"] = blk(xb, B, S, Lp).float().cpu().numpy()
        # row-parallel GEMMs in 4 row blocks, each all-reduce on a side stream
        blk4 = PX.TPBlock.from_full(full, heads, d, rank, world, chunks=4)
        res["block4"] = blk4(xb, B, S, Lp).float().cpu().numpy()
        torch.cuda.synchronize()
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
