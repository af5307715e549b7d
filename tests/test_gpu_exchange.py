"""Peer-store exchange of KV-page-sharded partials (exchange.cu).

Emulated on one GPU: W ranks' decodes run one after another, each pushing
its merged rows into W gather buffers that all live on this GPU (the same
kernels a multi-GPU run uses, with local addresses where peers' would be), so
no wait can depend on another launch still to come.  The merged output must
be the same on every rank, bit for bit, and equal the unsharded decode within
1e-3 (f32 partials merged in a different order); a second exchange checks the
counters that only grow.  A wait whose rows never arrive ends with the
exchange-timeout status and leaves the context usable.  With two or more
GPUs, the same exchange runs as one process per GPU over CUDA IPC mappings
(a gloo group only carries the IPC handles).
"""

import ctypes
import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import flagattention_b200 as fa
import oracle
from flagattention_b200 import _lib, shard
from flagattention_b200 import _torch as fat
from inputs import paged_pool
from mla_cases import D_QK, D_V, assert_close

pytestmark = pytest.mark.gpu

PAGE = 64
SCALE = D_QK ** -0.5


def _inputs(seed, lens, heads=128):
    bt, npages = paged_pool(lens, PAGE, seed + 1)
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((len(lens), 1, heads, D_QK), generator=g).to(torch.bfloat16).cuda()
    kc = torch.randn((npages, PAGE, 1, D_QK), generator=g).to(torch.bfloat16).cuda()
    return q, kc, bt


def _buffers(world, rows):
    """world gather buffers (f32 parts) and counter arrays, all on this GPU."""
    parts = [torch.zeros(world * rows * (D_V + 1), dtype=torch.float32, device="cuda")
             for _ in range(world)]
    cnts = [torch.zeros(world, dtype=torch.int64, device="cuda") for _ in range(world)]
    return parts, cnts


def _push_all(q, kc, bt, lens, world, parts, cnts):
    """Every emulated rank decodes its pages and pushes its rows."""
    keep = []
    arr_p = (ctypes.c_void_p * world)(*[p.data_ptr() for p in parts])
    arr_c = (ctypes.c_void_p * world)(*[c.data_ptr() for c in cnts])
    stream = fat.stream_of(q)
    for rank in range(world):
        lbt, llen = shard.shard_pages(bt, lens, PAGE, world, rank)
        pd = shard.PartialDecode(q, kc, torch.from_numpy(lbt).cuda(),
                                 torch.from_numpy(llen).cuda(), SCALE)
        keep.append(pd)
        _lib.check(_lib.lib().fa_mla_decode_partial(pd.call._ref, stream), "decode")
        _lib.check(_lib.lib().fa_mla_combine_push(pd.call._ref, arr_p, arr_c, world, rank,
                                                  stream), "push")
    return keep


def _merge(parts, cnts, rank, world, rows, target, timeout_ns=2_000_000_000, dtype=torch.float32):
    out = torch.full((rows, D_V), float("nan"), dtype=dtype, device="cuda")
    lse = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
    st = fat.status_word(out.device)
    _lib.check(_lib.lib().fa_lse_merge_wait(
        ctypes.c_void_p(parts[rank].data_ptr()), world, rows, D_V,
        ctypes.c_void_p(cnts[rank].data_ptr()), target, ctypes.c_void_p(out.data_ptr()),
        fat.dtype_code(out), ctypes.c_void_p(lse.data_ptr()), ctypes.c_void_p(st.data_ptr()),
        timeout_ns, fat.stream_of(out)), "merge wait")
    return out, lse


@pytest.mark.parametrize("world", [2, 3, 8])
def test_emulated_peer_exchange_matches_unsharded(world):
    lens = np.array([20000, 777, 64 * 40], np.int32)
    q, kc, bt = _inputs(80 + world, lens)
    B, h_q = len(lens), q.shape[2]
    rows = B * h_q
    full = torch.empty((B, 1, h_q, D_V), dtype=torch.float32, device="cuda")
    meta, splits = fa.get_mla_metadata(torch.from_numpy(lens).cuda(), h_q, 1)
    _, full_lse = fa.flash_mla_with_kvcache(q, kc, torch.from_numpy(bt).cuda(),
                                            torch.from_numpy(lens).cuda(), D_V, meta, splits,
                                            softmax_scale=SCALE, out=full)
    parts, cnts = _buffers(world, rows)
    for epoch in (1, 2):                       # counters keep growing across exchanges
        _push_all(q, kc, bt, lens, world, parts, cnts)
        outs = [_merge(parts, cnts, r, world, rows, epoch * rows) for r in range(world)]
        torch.cuda.synchronize()
        assert fat.read_status(q.device) == 0
        assert (cnts[0].cpu() == epoch * rows).all()
        for r in range(1, world):
            assert torch.equal(outs[r][0], outs[0][0]) and torch.equal(outs[r][1], outs[0][1])
        out0 = outs[0][0].view(B, 1, h_q, D_V)
        assert_close("out", out0.cpu().numpy(), full.cpu().numpy(), atol=1e-3, rtol=1e-3)
        assert_close("lse", outs[0][1].view(B, h_q, 1).cpu().numpy(), full_lse.cpu().numpy(),
                     atol=1e-3, rtol=1e-3)
    b = 1
    q_np = q.float().cpu().numpy()
    want_o, want_l = oracle.mla_decode_dense(q_np[b:b + 1], kc.float().cpu().numpy(),
                                             bt[b:b + 1], lens[b:b + 1], D_V, SCALE)
    assert_close("oracle out", out0[b:b + 1].cpu().numpy(), want_o)


def test_merge_wait_times_out_when_rows_never_arrive():
    """The counters never reach the target: the wait gives up after its time
    limit, writes nothing, reports the exchange timeout, and the context stays
    usable for the next decode."""
    world, rows = 2, 256
    parts, cnts = _buffers(world, rows)
    out, lse = _merge(parts, cnts, 0, world, rows, target=rows, timeout_ns=20_000_000)
    torch.cuda.synchronize()
    assert fat.read_status(out.device) == _lib.FA_DEVICE_TIMEOUT_EXCHANGE
    assert torch.isnan(out).all() and torch.isnan(lse).all()
    lens = np.array([300], np.int32)
    q, kc, bt = _inputs(91, lens)
    meta, splits = fa.get_mla_metadata(torch.from_numpy(lens).cuda(), 128, 1)
    o, l = fa.flash_mla_with_kvcache(q, kc, torch.from_numpy(bt).cuda(),
                                     torch.from_numpy(lens).cuda(), D_V, meta, splits,
                                     softmax_scale=SCALE)
    torch.cuda.synchronize()
    assert fat.read_status(q.device) == 0
    want_o, want_l = oracle.mla_decode_dense(q.float().cpu().numpy(), kc.float().cpu().numpy(),
                                             bt, lens, D_V, SCALE)
    assert_close("out after timeout", o.float().cpu().numpy(), want_o)


def _exchange(pd, parts, cnts, world, rank, rows, target, timeout_ns=2_000_000_000):
    """fa_mla_combine_exchange of one emulated rank: its merged output."""
    out = torch.full((rows, D_V), float("nan"), dtype=torch.bfloat16, device="cuda")
    lse = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
    st = fat.status_word(out.device)
    arr_p = (ctypes.c_void_p * world)(*[p.data_ptr() for p in parts])
    arr_c = (ctypes.c_void_p * world)(*[c.data_ptr() for c in cnts])
    _lib.check(_lib.lib().fa_mla_combine_exchange(
        pd.call._ref, arr_p, arr_c, world, rank, target, ctypes.c_void_p(out.data_ptr()),
        fat.dtype_code(out), ctypes.c_void_p(lse.data_ptr()), ctypes.c_void_p(st.data_ptr()),
        timeout_ns, fat.stream_of(out)), "exchange")
    return out, lse


def test_fused_exchange_with_emulated_peer():
    """The one-launch exchange (push, wait, merge) on this GPU: rank 1's rows
    are pushed first by the separate push kernel (which never waits), then
    rank 0's fused kernel pushes its own rows, finds both ranks' rows and
    merges; then rank 1's fused kernel does the same.  Both equal the
    unsharded decode."""
    world = 2
    lens = np.array([20000, 777, 64 * 40], np.int32)
    q, kc, bt = _inputs(95, lens)
    B, h_q = len(lens), q.shape[2]
    rows = B * h_q
    meta, splits = fa.get_mla_metadata(torch.from_numpy(lens).cuda(), h_q, 1)
    full, full_lse = fa.flash_mla_with_kvcache(q, kc, torch.from_numpy(bt).cuda(),
                                               torch.from_numpy(lens).cuda(), D_V, meta, splits,
                                               softmax_scale=SCALE)
    parts, cnts = _buffers(world, rows)
    pds = []
    for rank in range(world):
        lbt, llen = shard.shard_pages(bt, lens, PAGE, world, rank)
        pds.append(shard.PartialDecode(q, kc, torch.from_numpy(lbt).cuda(),
                                       torch.from_numpy(llen).cuda(), SCALE))
    stream = fat.stream_of(q)
    arr_p = (ctypes.c_void_p * world)(*[p.data_ptr() for p in parts])
    arr_c = (ctypes.c_void_p * world)(*[c.data_ptr() for c in cnts])
    L = _lib.lib()
    _lib.check(L.fa_mla_decode_partial(pds[1].call._ref, stream), "decode 1")
    _lib.check(L.fa_mla_combine_push(pds[1].call._ref, arr_p, arr_c, world, 1, stream), "push 1")
    _lib.check(L.fa_mla_decode_partial(pds[0].call._ref, stream), "decode 0")
    out0, lse0 = _exchange(pds[0], parts, cnts, world, 0, rows, rows)
    _lib.check(L.fa_mla_decode_partial(pds[1].call._ref, stream), "decode 1")
    out1, lse1 = _exchange(pds[1], parts, cnts, world, 1, rows, rows)
    torch.cuda.synchronize()
    assert fat.read_status(q.device) == 0
    assert torch.equal(out0, out1) and torch.equal(lse0, lse1)
    assert_close("out", out0.view(B, 1, h_q, D_V).float().cpu().numpy(),
                 full.float().cpu().numpy())
    assert_close("lse", lse0.view(B, h_q, 1).cpu().numpy(), full_lse.cpu().numpy())


def test_fused_exchange_times_out_without_peer():
    """A peer that never pushes: the fused kernel pushes its own rows, waits
    at most its time limit, merges nothing and reports the exchange timeout."""
    world = 2
    lens = np.array([3000], np.int32)
    q, kc, bt = _inputs(96, lens)
    rows = q.shape[2]
    parts, cnts = _buffers(world, rows)
    lbt, llen = shard.shard_pages(bt, lens, PAGE, world, 0)
    pd = shard.PartialDecode(q, kc, torch.from_numpy(lbt).cuda(), torch.from_numpy(llen).cuda(),
                             SCALE)
    _lib.check(_lib.lib().fa_mla_decode_partial(pd.call._ref, fat.stream_of(q)), "decode")
    out, lse = _exchange(pd, parts, cnts, world, 0, rows, rows, timeout_ns=20_000_000)
    torch.cuda.synchronize()
    assert fat.read_status(q.device) == _lib.FA_DEVICE_TIMEOUT_EXCHANGE
    assert torch.isnan(out.float()).all() and torch.isnan(lse).all()
    assert int(cnts[1][0].item()) == rows                  # its own rows did reach the peer


def _peer_worker(rank, world, port, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    try:
        torch.cuda.set_device(rank)
        shard.new_group_with_timeout("gloo", 60, rank=rank, world_size=world)
        lens = np.array([65536, 1000], np.int32)
        bt, npages = paged_pool(lens, PAGE, 71)
        g = torch.Generator().manual_seed(70)                       # same values on every rank
        q = torch.randn((2, 1, 128, D_QK), generator=g).to(torch.bfloat16).cuda()
        kc = torch.randn((npages, PAGE, 1, D_QK), generator=g).to(torch.bfloat16).cuda()
        lbt, llen = shard.shard_pages(bt, lens, PAGE, world, rank)
        dec = shard.PeerLongContextDecode(q, kc, torch.from_numpy(lbt).cuda(),
                                          torch.from_numpy(llen).cuda(), SCALE)
        for _ in range(2):                                          # exchanges in a row:
            out, lse = dec.run()                                    # fused push + merge
        dec.decode()
        dec.push()                                                  # and as two launches
        dec.merge()
        out, lse = dec.out, dec.lse
        torch.cuda.synchronize()
        status = fat.read_status(q.device)
        np.savez(os.path.join(outdir, f"rank{rank}.npz"), out=out.float().cpu().numpy(),
                 lse=lse.cpu().numpy(), status=status,
                 q=q.float().cpu().numpy() if rank == 0 else 0)
        torch.distributed.barrier()
        dec.close()
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    except Exception:
        with open(os.path.join(outdir, f"rank{rank}.err"), "w") as f:
            f.write(traceback.format_exc())
        raise


@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_exchange_multi_gpu(tmp_path, world):
    """One process per GPU: KV pages split over the ranks, partials exchanged
    by peer stores (no collective), every rank merges the same result."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_peer_worker, args=(r, world, port, str(tmp_path)))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    hung = [p for p in procs if p.is_alive()]
    for p in hung:
        p.kill()
        p.join(10)
    errs = [f.read_text() for f in tmp_path.glob("*.err")]
    assert not hung and all(p.exitcode == 0 for p in procs), errs
    z = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    for r in range(world):
        assert int(z[r]["status"]) == 0
        assert np.array_equal(z[0]["out"], z[r]["out"]) and np.array_equal(z[0]["lse"], z[r]["lse"])
    lens = np.array([65536, 1000], np.int32)
    bt, npages = paged_pool(lens, PAGE, 71)
    g = torch.Generator().manual_seed(70)
    torch.randn((2, 1, 128, D_QK), generator=g)
    kc = torch.randn((npages, PAGE, 1, D_QK), generator=g).to(torch.bfloat16).float().numpy()
    want_o, want_l = oracle.mla_decode_dense(z[0]["q"], kc, bt, lens, D_V, SCALE)
    assert_close("out", z[0]["out"], want_o)
    assert_close("lse", z[0]["lse"], want_l)
