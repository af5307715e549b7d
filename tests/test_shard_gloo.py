"""Host side of the multi-GPU sharding layer, on CPU ranks over gloo.

Covers ``flagattention_b200.shard``: the sequence partition used by batched
decode, the KV-page split used by long-context decode, the all-gather of
packed partials (O, LSE) between ranks, and a rank that fails before the exchange
(its peer must get an error within the group timeout, not hang).  The
per-rank decode here is the CPU oracle, so the merged result can be checked
against the oracle's unsharded decode.
"""

import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle
from flagattention_b200 import shard
from inputs import mla_inputs

D_V, PAGE = 512, 64
SCALE = 576 ** -0.5


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_partition_sequences_covers_and_balances():
    rs = np.random.RandomState(0)
    for world in (1, 2, 3, 8):
        lens = rs.randint(1, 30000, size=int(rs.randint(1, 300)))
        bins = shard.partition_sequences(lens, world)
        assert len(bins) == world
        flat = sorted(i for b in bins for i in b)
        assert flat == list(range(len(lens)))
        assert shard.partition_sequences(lens, world) == bins          # deterministic
        loads = [sum(int(lens[i]) for i in b) for b in bins]
        # longest-first greedy: the spread never exceeds the longest sequence
        assert max(loads) - min(loads) <= int(lens.max())


def test_shard_pages_tiles_each_sequence():
    rs = np.random.RandomState(1)
    lens = np.array([0, 1, 63, 64, 65, 1000, 4096, 777], np.int32)
    npg = -(-lens // PAGE)
    bt = np.full((len(lens), int(npg.max())), -7, np.int32)
    for b, k in enumerate(npg):
        bt[b, :k] = rs.permutation(10000)[:k]
    for world in (1, 2, 3, 8):
        got_tok = np.zeros_like(lens)
        pages = [[] for _ in lens]
        for rank in range(world):
            lbt, llen = shard.shard_pages(bt, lens, PAGE, world, rank)
            assert llen.dtype == np.int32 and lbt.dtype == np.int32
            for b in range(len(lens)):
                k = -(-int(llen[b]) // PAGE)
                pages[b].extend(lbt[b, :k].tolist())
                got_tok[b] += llen[b]
        assert np.array_equal(got_tok, lens)
        for b, k in enumerate(npg):
            assert pages[b] == bt[b, :k].tolist()                     # in order, no gaps


def _oracle_partial(q, kc, lbt, llen):
    """One rank's (O, LSE) from the oracle, laid out like decode_partial's."""
    o, lse = oracle.mla_decode_dense(q, kc, lbt, llen, D_V, SCALE)
    return torch.from_numpy(o), torch.from_numpy(np.ascontiguousarray(lse.transpose(0, 2, 1)))


def _exchange_worker(rank, world, port, lens, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        shard.new_group_with_timeout("gloo", 30, rank=rank, world_size=world)
        q, kc, bt = mla_inputs(33, len(lens), 1, 8, lens)
        lbt, llen = shard.shard_pages(bt, lens, PAGE, world, rank)
        part_o, part_lse = _oracle_partial(q, kc, lbt, llen)
        B, _, H, _ = part_o.shape
        packed = shard.packed_partial(B, H)
        o_view, l_view = shard.unpack_partial(packed, B, H)
        o_view.copy_(part_o)
        l_view.copy_(part_lse.transpose(1, 2))
        gathered = shard.exchange_partials(packed)
        assert gathered.shape == (world, packed.numel())
        all_o = gathered[:, :B * H * D_V].reshape((world,) + tuple(part_o.shape))
        all_l = gathered[:, B * H * D_V:].reshape((world,) + tuple(part_lse.shape))
        assert torch.equal(all_o[rank], part_o) and torch.equal(all_l[rank], part_lse)
        out, lse = oracle.lse_combine(all_o.numpy(), all_l.numpy())
        np.savez(os.path.join(outdir, f"rank{rank}.npz"), out=out, lse=lse)
        torch.distributed.destroy_process_group()
    except Exception:
        with open(os.path.join(outdir, f"rank{rank}.err"), "w") as f:
            f.write(traceback.format_exc())
        raise


def _run_ranks(fn, world, args, timeout=120):
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=fn, args=(r, world) + args) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
        p.join(10)
    assert not alive, "a rank did not finish in time"
    return [p.exitcode for p in procs]


@pytest.mark.parametrize("world", [2, 3])
def test_kv_page_sharded_exchange_matches_unsharded(tmp_path, world):
    lens = np.array([700, 64, 1, 300], np.int32)       # includes ranks holding nothing
    codes = _run_ranks(_exchange_worker, world, (_free_port(), lens, str(tmp_path)))
    errs = [f.read_text() for f in tmp_path.glob("*.err")]
    assert codes == [0] * world, errs
    q, kc, bt = mla_inputs(33, len(lens), 1, 8, lens)
    want_o, want_l = oracle.mla_decode_dense(q, kc, bt, lens, D_V, SCALE)
    for r in range(world):
        z = np.load(tmp_path / f"rank{r}.npz")
        np.testing.assert_allclose(z["out"], want_o, atol=1e-5, rtol=1e-5)
        np.testing.assert_allclose(z["lse"], want_l.transpose(0, 2, 1), atol=1e-5, rtol=1e-5)


def _failing_worker(rank, world, port, outdir):
    """Rank 1 raises before the exchange; rank 0 must see an error, not hang."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    shard.new_group_with_timeout("gloo", 5, rank=rank, world_size=world)
    if rank == 1:
        raise RuntimeError("injected failure on rank 1 before the exchange")
    packed = torch.zeros(shard.packed_partial(1, 4).numel())
    try:
        shard.exchange_partials(packed)
    except Exception as e:                               # the expected path
        with open(os.path.join(outdir, "rank0.caught"), "w") as f:
            f.write(type(e).__name__ + ": " + str(e)[:200])
        return
    with open(os.path.join(outdir, "rank0.completed"), "w") as f:
        f.write("exchange completed without its peer")


def test_dead_rank_ends_exchange_with_error(tmp_path):
    codes = _run_ranks(_failing_worker, 2, (_free_port(), str(tmp_path)), timeout=90)
    assert codes[1] != 0                                  # the injected failure
    assert (tmp_path / "rank0.caught").exists(), codes
    assert not (tmp_path / "rank0.completed").exists()
