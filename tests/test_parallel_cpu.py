"""The multi-GPU layer's host logic on CPU: gloo ranks (world size 2) with the
oracle test double standing in for the CUDA kernels.

Checks that (1) token-row shards quantized with the 4-byte global-amax all-reduce give
exactly the bytes and scale of the unsharded quantization; (2) the tensor-parallel
FFN and DiT block (column/row parallel FP8 linears, head-split attention, fp32
partial all-reduce) reproduce the single-rank result; (3) weight sharding helpers
cut the fused QKV weight by heads; (4) the sequence-parallel block (row shards in and
out) equals the replicated form."""
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
from oracle import oracle as O


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights(seed, heads=4, d=32, k=128, hidden=256):
    full = {}
    for i, (name, n, kk) in enumerate([("qkv", 3 * heads * d, k), ("out", k, heads * d), ("up", hidden, k),
                                       ("down", k, hidden)]):
        w = GI.randn_bf16(seed + i, (n, kk), 0.05)
        q, s = O.quantize_weight(w)
        b = GI.randn_bf16(seed + 10 + i, (n,), 0.1) if name in ("qkv", "out") else None
        full[name] = (torch.from_numpy(q).view(torch.float8_e4m3fn), torch.tensor([s]), b)
    return full


def _worker(rank, world, port, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from parallel_oracle_ops import OracleOps
        from qik import parallel as PX
        ops = OracleOps()
        res = {}
        # (1) sharded quantization with the global amax
        x = GI.outlier_activations(3, 97, 128)
        x[0, 0] = 1000.0                        # the global amax lives in rank 0's rows
        lo, hi = PX.row_range(x.shape[0], rank, world)
        q, s = PX.quantize_sharded(x[lo:hi].contiguous(), ops=ops)
        res["shard_q"] = (lo, hi, q.view(torch.uint8).numpy().copy(), float(s[0]))
        q2, s2 = PX.quantize_sharded(x[lo:hi].contiguous(), global_amax=False, ops=ops)
        res["shard_local_scale"] = float(s2[0])
        # (2) TP FFN and (3) TP block
        heads, d, k, hidden, B, S = 4, 32, 128, 256, 2, 24
        full = _weights(50, heads, d, k, hidden)
        blk = PX.TPBlock.from_full(full, heads, d, rank, world, ops=ops)
        xb = GI.randn_bf16(60, (B * S, k))
        Lp = torch.arange(S, dtype=torch.int32)
        Lp[4:] = S - 1
        res["ffn"] = PX.tp_ffn(xb, blk.up, blk.down).float().numpy()
        res["block"] = blk(xb, B, S, Lp).float().numpy()
        # (4) the sequence-parallel form: this rank's rows in and out
        sp = PX.TPBlock.from_full(full, heads, d, rank, world, ops=ops, sequence_parallel=True)
        lo, hi = rank * (B * S // world), (rank + 1) * (B * S // world)
        y_sp, amax_sp = sp.forward_sp(xb[lo:hi].contiguous(), B, S, Lp)
        res["block_sp"] = (lo, hi, y_sp.float().numpy(), int(amax_sp.reshape(-1)[0].item()))
        y2, _ = sp.forward_sp(y_sp, B, S, Lp, amax_sp)   # a second block fed the first one's amax
        res["block_sp2"] = y2.float().numpy()
        res["block2"] = blk(blk(xb, B, S, Lp), B, S, Lp).float().numpy()
        h_sp, _ = PX.tp_ffn_sp(xb[lo:hi].contiguous(), None, sp.up, sp.down)
        res["ffn_sp"] = h_sp.float().numpy()
        # row shards that do not split evenly are refused before any collective
        odd = torch.ones(2 * world + 1, 8)
        try:
            PX.reduce_scatter_rows(odd)
            res["uneven_refused"] = world == 1
        except ValueError:
            res["uneven_refused"] = world > 1
        # e4m3 rows gather as bytes, in rank order
        mine = torch.full((2, 4), float(rank + 1)).to(torch.float8_e4m3fn)
        res["gathered"] = PX.all_gather_rows(mine).float().numpy()
        with open(os.path.join(outdir, f"r{rank}.pkl"), "wb") as f:
            pickle.dump(res, f)
    finally:
        dist.destroy_process_group()


def _run(world):
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(world, _free_port(), d), nprocs=world, start_method="spawn", join=True)
        out = []
        for r in range(world):
            with open(os.path.join(d, f"r{r}.pkl"), "rb") as f:
                out.append(pickle.load(f))
        return out


@pytest.fixture(scope="module")
def results():
    return _run(1), _run(2)


def test_sharded_quantization_matches_unsharded(results):
    one, two = results
    lo, hi, q_full, s_full = one[0]["shard_q"]
    assert (lo, hi) == (0, 97)
    got = np.concatenate([r["shard_q"][2] for r in two], 0)
    assert np.array_equal(got, q_full)
    assert all(r["shard_q"][3] == s_full for r in two)
    # without the all-reduce, the shard that does not hold the global amax gets its own scale
    assert two[0]["shard_local_scale"] == s_full
    assert two[1]["shard_local_scale"] < s_full


def test_tp_ffn_matches_single_rank(results):
    one, two = results
    ref = torch.from_numpy(one[0]["ffn"])
    for r in two:
        y = torch.from_numpy(r["ffn"])
        assert O.relf(y, ref) <= 5e-3
        assert (y - ref).abs().max().item() <= 2e-2 + 0.01 * ref.abs().max().item()


def test_sequence_parallel_block_equals_replicated_form(results):
    """Row shards in and out (reduce-scatter, e4m3 all-gather with the global scale):
    the concatenated rows equal the replicated TP block's output bit for bit on the same
    ranks (the same sums; the same e4m3 bytes), two blocks in a row included, and the
    returned amax is max|output| of the rank's rows."""
    for runs in results:
        for r in runs:
            lo, hi, y, amax_bits = r["block_sp"]
            assert np.array_equal(y, r["block"][lo:hi])
            assert amax_bits == int(np.float32(np.abs(y).max()).view(np.int32))
            assert np.array_equal(r["block_sp2"], r["block2"][lo:hi])
            assert np.array_equal(r["ffn_sp"], r["ffn"][lo:hi])


def test_sequence_parallel_helpers(results):
    """reduce_scatter_rows refuses rows that do not split over the ranks (and is the
    identity on one rank); all_gather_rows concatenates e4m3 shards in rank order."""
    for runs in results:
        world = len(runs)
        for r in runs:
            assert r["uneven_refused"]
            want = np.concatenate([np.full((2, 4), float(k + 1), dtype=np.float32) for k in range(world)], 0)
            assert np.array_equal(r["gathered"], want)


def test_tp_block_matches_single_rank(results):
    one, two = results
    ref = torch.from_numpy(one[0]["block"])
    for r in two:
        y = torch.from_numpy(r["block"])
        assert O.relf(y, ref) <= 5e-3


def test_qkv_head_sharding_layout():
    from qik import parallel as PX
    heads, d, k = 4, 8, 16
    w = torch.arange(3 * heads * d * k, dtype=torch.float32).reshape(3 * heads * d, k)
    for world in (1, 2, 4):
        parts = [PX.shard_qkv_heads(w, heads, d, r, world) for r in range(world)]
        hl = heads // world
        for r, p in enumerate(parts):
            for j in range(3):
                exp = w[j * heads * d + r * hl * d: j * heads * d + (r + 1) * hl * d]
                assert torch.equal(p[j * hl * d:(j + 1) * hl * d], exp)
    with pytest.raises(ValueError):
        PX.shard_qkv_heads(w, heads, d, 0, 3)
    assert PX.row_range(10, 0, 3) == (0, 4) and PX.row_range(10, 2, 3) == (7, 10)
