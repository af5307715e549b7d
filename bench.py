#!/usr/bin/env python
"""MLA decode benchmark on B200 (one JSON line on rank 0).

Headline workload: DeepSeek-V3-shaped dense paged MLA
decode -- 64 sequences per GPU, seq_q 1, 128 query heads, one 576-dim latent
head (values = first 512 dims), page 64, bf16 N(0,1), context lengths
U[1024, 8192], block table a random permutation of a pooled page cache,
softmax scale 576^-0.5.  A step is one decode of the batch (decode kernel,
which merges short splits itself, + the combine kernel for long ones, queued
as its programmatic dependent; the tile metadata is computed once per batch,
as it is shared by every layer of a model step).  With --gpus N (torchrun) the global batch
of 64*N sequences is sharded by sequence across the ranks (greedy by KV bytes,
no collective on the data path): weak scaling.

The same line carries ``long_context``: BASELINE config 5 (2 sequences of
1,048,576 tokens) with the KV pages split evenly over the N ranks -- strong
scaling.  Each rank decodes its pages; one cooperative kernel merges its
split pieces, stores every row into every rank's gather buffer over NVLink
(peer stores, no collective), waits for all ranks' rows and merges them.  The
same step with one NCCL all-gather of packed partials is timed beside it.

Inputs of sequence i (query and its KV rows) come from a CPU generator seeded
with i, so both arms decode the same values.  ``--impl reference`` times the
reference algorithm's CPU implementation (the numpy restatement of
flag_attn.testing in oracle/) on all host cores, on the first sequences of the
same global batch.
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

B_PER_GPU, S_Q, H_Q, D_QK, D_V, PAGE = 64, 1, 128, 576, 512, 64
CTX_LO, CTX_HI = 1024, 8192
SEED = 2026
WORKLOAD = "dense_paged_mla_decode_b64_h128_ctx1k-8k_bf16"
METRIC = "mla_decode_tokens_per_s"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--cpu-seconds", type=float, default=10.0,
                   help="budget of the cpu_baseline sample")
    p.add_argument("--config", type=int, default=2, choices=[2, 3, 4, 5],
                   help="BASELINE config; 2 is the headline workload, 3-5 are timed on one "
                        "GPU for the record (MTP causal, sparse top-k, 1M-token context)")
    p.add_argument("--batch", type=int, default=0,
                   help="configs 3-5: first N sequences only (smaller cases for profiling)")
    p.add_argument("--gqa", default=None, metavar="KEY=VALUE,...",
                   help="time only the grouped-query paged_attention record on one GPU, its "
                        "shape changed by overrides (keys: seqs, heads_q, heads_kv, head, "
                        "page, ctx, splits); '' keeps the default shape")
    return p.parse_args()


def global_lens(world):
    rs = np.random.RandomState(SEED)
    return rs.randint(CTX_LO, CTX_HI + 1, size=B_PER_GPU * world).astype(np.int32)


def sequence_inputs(i, n):
    """Query [S_Q, H_Q, 576] and KV rows [pages*64, 576] (bf16) of global
    sequence i with context n, from a CPU generator seeded with i: the same
    values in both arms, at every GPU count."""
    import torch
    g = torch.Generator().manual_seed(SEED * 1000 + int(i))
    q = torch.randn((S_Q, H_Q, D_QK), generator=g).to(torch.bfloat16)
    kv = torch.randn((-(-int(n) // PAGE) * PAGE, D_QK), generator=g).to(torch.bfloat16)
    return q, kv


def config_dict(world):
    return {"workload": WORKLOAD, "batch_per_gpu": B_PER_GPU, "global_batch": B_PER_GPU * world,
            "seq_q": S_Q, "heads_q": H_Q, "d_qk": D_QK, "d_v": D_V, "page_size": PAGE,
            "ctx": [CTX_LO, CTX_HI], "parallelism": f"seq-shard{world}",
            "inputs": "sequence i from a CPU torch generator seeded with i (bf16 N(0,1))",
            "l2": "flushed before every step (256 MB write, outside the events)",
            "metadata": "computed once per batch (outside the step)"}


def algorithmic_bytes(lens):
    n = len(lens)
    return int(np.sum(lens.astype(np.int64)) * D_QK * 2 + n * S_Q * H_Q * (D_QK * 2 + D_V * 2 + 4))


def algorithmic_flops(lens):
    return int(np.sum(lens.astype(np.int64)) * 2 * S_Q * H_Q * (D_QK + D_V))


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:  # noqa: BLE001
        return 6650.0, 1590.0, "fallback"


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """SM clock and clock-event reasons of one GPU, sampled during the timed
    region.  NVML (read-only queries) from a background thread every 2 ms,
    so even a timed region of a few tens of milliseconds gets samples;
    nvidia-smi is the fallback when NVML is missing."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))
    SMI_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                  "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                  "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, bus_id):
        self.sm, self.reasons, self.max_mhz = [], set(), None
        self.proc = self.thread = None
        try:
            import threading

            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus_id)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
            self.stop_evt = threading.Event()
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
        except Exception:
            self.thread = None
            self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            try:
                self.proc = subprocess.Popen(
                    ["nvidia-smi", f"--query-gpu={self.SMI_FIELDS}", "--format=csv,noheader,nounits",
                     "-lms", "100", "-i", bus_id], stdout=self.tmp, stderr=subprocess.DEVNULL)
            except OSError:
                self.proc = None

    def _poll(self):
        nv = self.nvml
        while not self.stop_evt.is_set():
            try:
                self.sm.append(float(nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)))
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                for name, const in self.REASONS:
                    if mask & getattr(nv, const, 0):
                        self.reasons.add(name)
            except Exception:
                pass
            self.stop_evt.wait(0.002)

    def stop(self):
        if self.thread is not None:
            self.stop_evt.set()
            self.thread.join(timeout=5)
            return {"sm_mhz": statistics.median(self.sm) if self.sm else None,
                    "sm_max_mhz": float(self.max_mhz) if self.max_mhz else None,
                    "reasons": sorted(self.reasons), "samples": len(self.sm), "source": "nvml"}
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait(timeout=10)
        self.tmp.flush()
        rows = [r.split(",") for r in open(self.tmp.name).read().strip().splitlines() if r]
        os.unlink(self.tmp.name)
        sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) >= 9 and r[2].strip().replace(".", "").isdigit()]
        reasons = set()
        for r in rows:
            if len(r) >= 9:
                for (name, _), val in zip(self.REASONS, r[5:9]):
                    if val.strip() == "Active":
                        reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvidia-smi"}


# ---------------------------------------------------------------- our arm
def build_batch(lens, gidx, dev):
    """Paged pool (pages in a random permutation) holding the sequences
    gidx (global indices, context lens), queries, block table."""
    import torch
    B = len(lens)
    npg = (lens + PAGE - 1) // PAGE
    npages = int(npg.sum())
    kcache = torch.empty((npages, PAGE, 1, D_QK), dtype=torch.bfloat16, device=dev)
    q = torch.empty((B, S_Q, H_Q, D_QK), dtype=torch.bfloat16, device=dev)
    perm = np.random.RandomState(SEED + 1 + int(gidx[0]) if B else SEED).permutation(npages)
    bt_np = np.zeros((B, int(npg.max())), np.int32)
    off = 0
    for j, (gi, n) in enumerate(zip(gidx, lens)):
        k = int(npg[j])
        pages = perm[off:off + k]
        off += k
        bt_np[j, :k] = pages
        qs, kv = sequence_inputs(gi, n)
        q[j] = qs.to(dev)
        kcache[torch.from_numpy(pages.astype(np.int64)).to(dev)] = \
            kv.view(k, PAGE, 1, D_QK).to(dev)
    return q, kcache, torch.from_numpy(bt_np).to(dev), npages


def run_ours(args):
    import torch
    import torch.distributed as dist

    import flagattention_b200 as fa
    from flagattention_b200 import _torch as fat
    from flagattention_b200.mla import MlaCall
    from flagattention_b200.shard import partition_sequences

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    lens_all = global_lens(world)
    mine = partition_sequences(lens_all, world)[rank]
    lens = lens_all[mine]
    B = len(lens)
    q, kcache, bt, npages = build_batch(lens, mine, dev)
    seq = torch.from_numpy(lens).to(dev)
    meta, splits = fa.get_mla_metadata(seq, S_Q * H_Q, 1)
    out = torch.empty((B, S_Q, H_Q, D_V), dtype=torch.bfloat16, device=dev)
    lse = torch.empty((B, H_Q, S_Q), dtype=torch.float32, device=dev)
    call = MlaCall(q, kcache, kcache.stride(0), kcache.stride(1), npages, PAGE, bt, seq, 0, meta,
                   splits, out, lse, D_QK ** -0.5)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)   # > 126 MB L2
    stream = torch.cuda.current_stream(dev)

    def step(ev):
        flush.fill_(1)
        ev[0].record(stream)
        call.run()          # decode kernel, then the combine queued as its dependent
        ev[1].record(stream)

    def decode_only(ev):
        flush.fill_(1)
        ev[0].record(stream)
        call.partial()      # the decode kernel alone
        ev[1].record(stream)

    for _ in range(args.warmup):
        step([torch.cuda.Event(enable_timing=True) for _ in range(2)])
        decode_only([torch.cuda.Event(enable_timing=True) for _ in range(2)])
    torch.cuda.synchronize()
    assert fat.read_status(dev) == 0, "device wait timeout during warm-up"

    props = torch.cuda.get_device_properties(dev)
    bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
    sampler = ClockSampler(bus) if rank == 0 else None
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    for i in range(args.steps):
        step(evs[i])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop() if sampler else None
    step_ms = sum(e[0].elapsed_time(e[1]) for e in evs) / args.steps
    dec_evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    for i in range(args.steps):
        decode_only(dec_evs[i])
    torch.cuda.synchronize()
    dec_ms = sum(e[0].elapsed_time(e[1]) for e in dec_evs) / args.steps
    assert fat.read_status(dev) == 0, "device wait timeout in the timed region"

    # end-to-end through the public API with host buffers
    q_h = q.cpu().pin_memory()
    seq_h = seq.cpu().pin_memory()
    bt_h = bt.cpu().pin_memory()
    q_d, seq_d, bt_d = torch.empty_like(q), torch.empty_like(seq), torch.empty_like(bt)
    out_h = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    lse_h = torch.empty(lse.shape, dtype=lse.dtype, pin_memory=True)

    def e2e_step(ev):
        flush.fill_(1)
        ev[0].record(stream)
        q_d.copy_(q_h, non_blocking=True)
        seq_d.copy_(seq_h, non_blocking=True)
        bt_d.copy_(bt_h, non_blocking=True)
        m, s = fa.get_mla_metadata(seq_d, S_Q * H_Q, 1)
        o, l = fa.flash_mla_with_kvcache(q_d, kcache, bt_d, seq_d, D_V, m, s)
        out_h.copy_(o, non_blocking=True)
        lse_h.copy_(l, non_blocking=True)
        ev[1].record(stream)

    for _ in range(args.warmup):
        e2e_step([torch.cuda.Event(enable_timing=True) for _ in range(2)])
    e2e_evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    for i in range(args.steps):
        e2e_step(e2e_evs[i])
    torch.cuda.synchronize()
    e2e_ms = sum(e[0].elapsed_time(e[1]) for e in e2e_evs) / args.steps
    # the end-to-end path computed the same outputs as the device-resident one
    call.run()
    torch.cuda.synchronize()
    assert torch.equal(out_h, out.cpu()) and torch.equal(lse_h, lse.cpu()), \
        "end-to-end output differs from the device-resident decode"
    h2d = q.numel() * 2 + seq.numel() * 4 + bt.numel() * 4
    d2h = out.numel() * 2 + lse.numel() * 4

    t = torch.tensor([step_ms, dec_ms, e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_ms, dec_ms, e2e_ms = t.tolist()

    # the HBM-bound records first: the tensor-heavy config-3 run leaves the
    # GPU near its power cap for a while
    gqa = run_gqa(args, dev, flush)
    long_ctx = run_long_context(args, world, rank, dev, flush)
    mtp = run_mtp_sharded(args, world, rank, dev, flush)

    tokens = len(lens_all) * S_Q
    bytes_local = algorithmic_bytes(lens)
    flops_local = algorithmic_flops(lens)
    if rank == 0:
        peak_gbs, peak_tf, peak_kind = measured_peaks()
        achieved = bytes_local / (dec_ms * 1e-3) / 1e9
        rec = {
            "metric": METRIC, "value": tokens / (step_ms * 1e-3), "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) bf16)",
            "config": config_dict(world),
            "hbm_gbs_step": bytes_local / (step_ms * 1e-3) / 1e9,
            "hbm_frac_step": bytes_local / (step_ms * 1e-3) / 1e9 / peak_gbs,
            "tensor_tflops_decode": flops_local / (dec_ms * 1e-3) / 1e12,
            "ms_decode_kernel": dec_ms,
            "ms_decode_kernel_note": "decode kernel timed alone in a second pass",
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak_gbs,
                         "unit": "GB/s", "frac": achieved / peak_gbs,
                         "traffic": None, "peak_source": peak_kind,
                         "kernel": "sv::mla_decode_sv_kernel<bf16> (score/value CTA pair)",
                         "algorithmic_bytes_per_launch": bytes_local},
            "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": "tok/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms,
                    "path": "get_mla_metadata + flash_mla_with_kvcache, pinned host buffers"},
            "gpu_launches": 2 * args.steps,
            "launches_per_step": "decode kernel + combine kernel (programmatic dependent launch; "
                                 "its blocks exit when every split was merged in the decode)",
            "clocks": clocks,
            "long_context": long_ctx,
            "mtp_causal": mtp,
            "gqa_paged": gqa,
        }
        if world == 1:
            rec["cpu_baseline"] = cpu_baseline(lens_all, args.cpu_seconds)
        print(json.dumps(rec), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------- config 5: KV pages over N ranks
LC_TOKENS, LC_BATCH = 1 << 20, 2
LC_WORKLOAD = "long_context_mla_decode_b2_h128_ctx1m_bf16_kv_page_sharded"


def run_long_context(args, world, rank, dev, flush):
    """BASELINE config 5 with the KV pages of both 1M-token sequences split
    evenly over the ranks (strong scaling).  A step: the decode of this
    rank's pages; one cooperative kernel that merges its split pieces, stores
    every row into every rank's gather buffer over NVLink, waits for all ranks'
    rows and merges them.  The same step with one NCCL all-gather of
    packed partials (decode + combine, all-gather, merge) is timed beside it.
    At N = 1 the step is the plain decode (+ combine) to bf16.  Every phase is
    timed with CUDA events on the launching stream; every figure (each phase,
    and the whole step of a rank) is the max over ranks."""
    import torch
    import torch.distributed as dist

    import flagattention_b200 as fa
    from flagattention_b200 import _torch as fat
    from flagattention_b200 import shard
    from flagattention_b200.mla import MlaCall

    pages_per_seq = LC_TOKENS // PAGE
    lo, hi = shard.page_range(pages_per_seq, world, rank)
    local_pages = hi - lo
    local_len = min(LC_TOKENS, hi * PAGE) - lo * PAGE
    g = torch.Generator(device=dev).manual_seed(SEED + 5000 + rank)
    pool = torch.empty((LC_BATCH * local_pages, PAGE, 1, D_QK), dtype=torch.bfloat16, device=dev)
    for a in range(0, pool.shape[0], 8192):
        b = min(pool.shape[0], a + 8192)
        pool[a:b] = torch.randn((b - a, PAGE, 1, D_QK), generator=g, device=dev)
    bt = torch.randperm(pool.shape[0], generator=g, device=dev).to(torch.int32)
    bt = bt.view(LC_BATCH, local_pages).contiguous()
    seq = torch.full((LC_BATCH,), local_len, dtype=torch.int32, device=dev)
    gq = torch.Generator(device=dev).manual_seed(SEED + 5999)          # same q on every rank
    q = torch.randn((LC_BATCH, 1, H_Q, D_QK), generator=gq, device=dev).to(torch.bfloat16)
    rows = LC_BATCH * H_Q
    stream = torch.cuda.current_stream(dev)

    def timed(step, n_ev):
        for _ in range(args.warmup):
            step([torch.cuda.Event(enable_timing=True) for _ in range(n_ev)])
        torch.cuda.synchronize()
        assert fat.read_status(dev) == 0, "device wait timeout during warm-up (long context)"
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(n_ev)] for _ in range(steps)]
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        for i in range(steps):
            step(evs[i])
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        assert fat.read_status(dev) == 0, "device wait timeout in the timed region (long context)"
        # per phase, and the whole step (first to last event) of this rank;
        # each the max over ranks.  The step's max is not the sum of the
        # phases' maxima: a rank whose decode ends early waits longer in the
        # exchange for the others.
        t = torch.tensor([sum(e[k].elapsed_time(e[k + 1]) for e in evs) / steps
                          for k in range(n_ev - 1)] +
                         [sum(e[0].elapsed_time(e[n_ev - 1]) for e in evs) / steps],
                         dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    steps = max(3, min(args.steps, 100))
    extra = {}
    if world == 1:
        meta, splits = fa.get_mla_metadata(seq, H_Q, 1)
        out = torch.empty((LC_BATCH, 1, H_Q, D_V), dtype=torch.bfloat16, device=dev)
        lse = torch.empty((LC_BATCH, H_Q, 1), dtype=torch.float32, device=dev)
        call = MlaCall(q, pool, pool.stride(0), pool.stride(1), pool.shape[0], PAGE, bt, seq, 0,
                       meta, splits, out, lse, D_QK ** -0.5)

        def step(ev):
            flush.fill_(1)
            ev[0].record(stream)
            call.run()
            ev[1].record(stream)

        dec_ms, step_ms = timed(step, 2)
        xchg_ms = None
        launches = 2
    else:
        # the product path: partials exchanged by peer stores (no collective)
        peer = shard.PeerLongContextDecode(q, pool, bt, seq, D_QK ** -0.5)

        def step(ev):
            flush.fill_(1)
            ev[0].record(stream)
            peer.decode()
            ev[1].record(stream)
            peer.exchange()
            ev[2].record(stream)

        dec_ms, xchg_ms, step_ms = timed(step, 3)
        launches = 2
        # for comparison: the same step with one NCCL all-gather of packed partials
        part = shard.PartialDecode(q, pool, bt, seq, D_QK ** -0.5)
        gathered = torch.empty((world, part.packed.numel()), dtype=torch.float32, device=dev)

        def step_nccl(ev):
            flush.fill_(1)
            ev[0].record(stream)
            part.call.run()
            ev[1].record(stream)
            dist.all_gather_into_tensor(gathered.view(-1), part.packed)
            ev[2].record(stream)
            shard.merge_partials(gathered, rows, D_V, torch.bfloat16)
            ev[3].record(stream)

        n_dec, n_gather, n_merge, n_step = timed(step_nccl, 4)
        extra = {"nccl_allgather_path": {"ms_per_step": n_step,
                                         "ms_decode_and_combine": n_dec,
                                         "us_allgather": n_gather * 1e3, "us_merge": n_merge * 1e3}}
        dist.barrier()
        peer.close()
        dist.barrier()
    peak_gbs, _, peak_kind = measured_peaks()
    kv_bytes = LC_BATCH * local_len * D_QK * 2 + rows * (D_QK * 2 + D_V * 4 + 4)
    rec = {"workload": LC_WORKLOAD, "baseline_config": 5, "n_gpus": world,
           "scaling": "strong", "steps": steps,
           "tokens_per_s": LC_BATCH / (step_ms * 1e-3), "ms_per_step": step_ms,
           "ms_decode": dec_ms,
           "us_exchange": xchg_ms * 1e3 if xchg_ms is not None else None,
           "exchange": ("one cooperative kernel: merge this rank's split pieces, store every "
                        "row into every rank's gather buffer over NVLink (peer stores), "
                        "bounded wait for all ranks' rows, merge (no collective)"
                        if world > 1 else None),
           "gpu_launches_per_step": launches,
           "exchange_bytes_per_rank": rows * (D_V + 1) * 4 * (world - 1) if world > 1 else 0,
           "tokens_per_rank": LC_BATCH * local_len,
           "hbm_frac_decode": kv_bytes / (dec_ms * 1e-3) / 1e9 / peak_gbs,
           "peak_source": peak_kind}
    rec.update(extra)
    return rec


# ------------------------- config 3: MTP causal, sequences over N ranks
def run_mtp_sharded(args, world, rank, dev, flush):
    """BASELINE config 3 (128 sequences, s_q = 2 causal, ctx log-uniform
    [4096, 32768]) with the sequences split over the ranks by KV bytes (no
    collective): strong scaling of the fixed batch.  A step: metadata-shared
    decode + combine of this rank's sequences; max over ranks."""
    import torch
    import torch.distributed as dist

    import flagattention_b200 as fa
    from flagattention_b200 import _torch as fat
    from flagattention_b200.mla import MlaCall
    from flagattention_b200.shard import partition_sequences

    lens_all = other_lens(3)
    mine = partition_sequences(lens_all, world)[rank]
    lens = lens_all[mine]
    B, s_q = len(lens), 2
    g = torch.Generator(device=dev).manual_seed(SEED + 300 + rank)
    npg = (lens + PAGE - 1) // PAGE
    npages = int(npg.sum())
    kc = torch.empty((npages, PAGE, 1, D_QK), dtype=torch.bfloat16, device=dev)
    for a in range(0, npages, 8192):
        b = min(npages, a + 8192)
        kc[a:b] = torch.randn((b - a, PAGE, 1, D_QK), generator=g, device=dev)
    q = torch.randn((B, s_q, H_Q, D_QK), generator=g, device=dev).to(torch.bfloat16)
    perm = torch.randperm(npages, generator=g, device=dev).to(torch.int32)
    bt = torch.zeros((B, int(npg.max())), dtype=torch.int32, device=dev)
    off = 0
    for i, k in enumerate(npg):
        bt[i, :k] = perm[off:off + int(k)]
        off += int(k)
    seq = torch.from_numpy(lens).to(dev)
    meta, splits = fa.get_mla_metadata(seq, s_q * H_Q, 1)
    out = torch.empty((B, s_q, H_Q, D_V), dtype=torch.bfloat16, device=dev)
    lse = torch.empty((B, H_Q, s_q), dtype=torch.float32, device=dev)
    call = MlaCall(q, kc, kc.stride(0), kc.stride(1), npages, PAGE, bt, seq, 0, meta, splits,
                   out, lse, D_QK ** -0.5, causal=True)
    stream = torch.cuda.current_stream(dev)
    steps = max(3, min(args.steps, 20))
    for _ in range(args.warmup):
        flush.fill_(1)
        call.run()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    for a, b in evs:
        flush.fill_(1)
        a.record(stream)
        call.run()
        b.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    assert fat.read_status(dev) == 0, "device wait timeout (config 3)"
    t = torch.tensor([sum(a.elapsed_time(b) for a, b in evs) / steps], dtype=torch.float64,
                     device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_ms = float(t.item())
    flops = int(np.sum(lens_all.astype(np.int64))) * 2 * s_q * H_Q * (D_QK + D_V)
    _, peak_tf, peak_kind = measured_peaks()
    return {"workload": OTHER[3]["workload"], "baseline_config": 3, "n_gpus": world,
            "scaling": "strong", "parallelism": f"seq-shard{world}", "steps": steps,
            "global_batch": len(lens_all), "seq_q": s_q, "causal": True,
            "tokens_per_s": len(lens_all) * s_q / (step_ms * 1e-3), "ms_per_step": step_ms,
            "gpu_launches_per_step": 2,
            "tensor_tflops_all_gpus": flops / (step_ms * 1e-3) / 1e12,
            "tensor_frac_per_gpu": flops / (step_ms * 1e-3) / 1e12 / world / peak_tf,
            "peak_source": peak_kind}


# ------------------ the reference's own paged API at a GQA shape (per GPU)
GQA = dict(seqs=32, heads_q=64, heads_kv=8, head=128, page=16, ctx=4096, splits=0)


def gqa_shape(spec):
    """GQA with the overrides of a `--gqa` value ("head=256,page=128")."""
    c = dict(GQA)
    for item in filter(None, (spec or "").split(",")):
        key, _, val = item.partition("=")
        if key not in c:
            raise SystemExit(f"--gqa: unknown key {key!r} (keys: {', '.join(c)})")
        c[key] = int(val)
    return c


def run_gqa(args, dev, flush, c=GQA):
    """`paged_attention` (paged.py:20) at a grouped-query shape: by default
    32 sequences of 4096 tokens, 64 query heads over 8 kv heads (group 8),
    head size 128, 16-token pages in a random permutation, bf16, the balanced
    schedule (num_splits 0).  Per GPU (each rank runs its own).  Bytes: every
    K and V row once + Q + O."""
    import torch

    import flagattention_b200 as fa
    from flagattention_b200 import _torch as fat

    g = torch.Generator(device=dev).manual_seed(SEED + 400)
    pages_per = c["ctx"] // c["page"]
    npages = c["seqs"] * pages_per
    shape = (npages, c["heads_kv"], c["page"], c["head"])
    kc = torch.randn(shape, generator=g, device=dev).to(torch.bfloat16)
    vc = torch.randn(shape, generator=g, device=dev).to(torch.bfloat16)
    q = torch.randn((c["seqs"], c["heads_q"], c["head"]), generator=g, device=dev).to(torch.bfloat16)
    bt = torch.randperm(npages, generator=g, device=dev).to(torch.int32).view(c["seqs"], -1)
    lens = torch.full((c["seqs"],), c["ctx"], dtype=torch.int32, device=dev)
    scale = c["head"] ** -0.5
    stream = torch.cuda.current_stream(dev)

    def step():
        return fa.paged_attention(q, kc, vc, lens, bt, scale, c["ctx"], c["splits"])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # K and V (537 MB) exceed L2 (126 MB): the calls run back to back between
    # two events, after the flush, so host-side argument handling overlaps
    # the previous call on the device instead of being timed as idle GPU
    steps = max(3, min(args.steps, 50))
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    flush.fill_(1)
    a.record(stream)
    for _ in range(steps):
        step()
    b.record(stream)
    torch.cuda.synchronize()
    assert fat.read_status(dev) == 0
    ms = a.elapsed_time(b) / steps
    nbytes = 2 * kc.numel() * 2 + 2 * q.numel() * 2
    peak_gbs, _, peak_kind = measured_peaks()
    name = "gqa_paged_decode_b{seqs}_hq{heads_q}_hkv{heads_kv}_d{head}_page{page}_ctx{ctx}_bf16"
    if c["splits"]:
        name += "_splits{splits}"
    return {"workload": name.format(**c),
            "api": "paged_attention (paged.py:20)", "steps": steps, "ms_per_step": ms,
            "l2": "inputs larger than L2, calls back to back",
            "tokens_per_s": c["seqs"] / (ms * 1e-3),
            "roofline": {"bound": "hbm", "achieved": nbytes / (ms * 1e-3) / 1e9,
                         "peak": peak_gbs, "unit": "GB/s",
                         "frac": nbytes / (ms * 1e-3) / 1e9 / peak_gbs,
                         "algorithmic_bytes": nbytes, "peak_source": peak_kind},
            "kernel": "gqa_decode_kernel (tcgen05, per-CTA balanced share) + merge of split entries"}


# ------------------------------------------------------------ CPU timing
def reference_samples(lens_all, n_seq):
    """The first n_seq sequences of the global batch as float32 numpy, each
    in a pool of exactly its pages (the same bf16 values the GPU arm decodes,
    upcast as the reference's fp32 path does)."""
    samples = []
    for i in range(min(n_seq, len(lens_all))):
        n = int(lens_all[i])
        qs, kv = sequence_inputs(i, n)
        k = (n + PAGE - 1) // PAGE
        samples.append((qs.float().numpy()[None], kv.float().numpy().reshape(k, PAGE, 1, D_QK),
                        np.arange(k, dtype=np.int32)[None], lens_all[i:i + 1]))
    return samples


def time_oracle(samples, budget_s):
    """Run the oracle over the samples round-robin for ~budget_s; tok/s."""
    import oracle
    done, t0 = 0, time.perf_counter()
    while True:
        qs, kc, bt, ln = samples[done % len(samples)]
        oracle.mla_decode_dense(qs, kc, bt, ln, D_V, D_QK ** -0.5)
        done += 1
        el = time.perf_counter() - t0
        if el >= budget_s and done >= 2:
            return done * S_Q / el, done, el


def all_host_threads():
    """Let BLAS use every host core, whatever the launcher set
    (torchrun exports OMP_NUM_THREADS=1); returns the thread count."""
    n = os.cpu_count() or 1
    from threadpoolctl import threadpool_limits
    threadpool_limits(limits=n)
    return n


def cpu_baseline(lens_all, budget):
    cores = all_host_threads()
    samples = reference_samples(lens_all, 8)
    tps, done, el = time_oracle(samples, budget)
    return {"value": tps, "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"{done} sequence decodes of the config-2 workload (global sequences 0-7, "
                      f"ctx {int(lens_all[:8].min())}-{int(lens_all[:8].max())}, 128 heads) "
                      f"through the numpy oracle in {el:.1f}s, float32, {cores} BLAS threads"}


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if int(os.environ.get("RANK", "0")) != 0:
        return
    cores = all_host_threads()
    lens_all = global_lens(world)
    n_seq = 8
    samples = reference_samples(lens_all, n_seq)
    per_step = max(0.5, min(2.0, 150.0 / max(1, args.steps + args.warmup)))
    for _ in range(args.warmup):
        time_oracle(samples, per_step)
    t0 = time.perf_counter()
    total_done = 0
    for _ in range(args.steps):
        _, d, _ = time_oracle(samples, per_step)
        total_done += d
    el = time.perf_counter() - t0
    value = total_done * S_Q / el
    rec = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3,
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
           "data": "synthetic (seeded N(0,1) bf16)", "impl": "reference",
           "config": config_dict(world),
           "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": "port",
                            "sample": f"each step decodes global sequences 0-{n_seq - 1} of the "
                                      f"config-2 batch (round-robin, ~{per_step:.1f}s) through "
                                      "the numpy restatement of flag_attn.testing, float32 "
                                      "upcast of the same bf16 inputs the GPU arm decodes"},
           "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}}
    print(json.dumps(rec), flush=True)


# ------------------------------------------------- configs 3-5 (one GPU)
OTHER = {
    3: dict(workload="mtp_causal_paged_mla_decode_b128_sq2_h128_ctx4k-32k-log_bf16",
            B=128, s_q=2, causal=True, topk=0),
    4: dict(workload="sparse_top2048_mla_decode_b64_h128_ctx32k-128k_bf16",
            B=64, s_q=1, causal=False, topk=2048),
    5: dict(workload="long_context_mla_decode_b2_h128_ctx1m_bf16",
            B=2, s_q=1, causal=False, topk=0),
}


def other_lens(cfg):
    rs = np.random.RandomState(SEED + cfg)
    if cfg == 3:
        return np.exp(rs.uniform(np.log(4096), np.log(32768), size=128)).astype(np.int32)
    if cfg == 4:
        return rs.randint(32768, 131073, size=64).astype(np.int32)
    return np.array([1 << 20, 1 << 20], np.int32)


def run_other(args):
    """Decode + combine step of BASELINE config 3, 4 or 5 on one GPU: seeded
    N(0,1) bf16 inputs made on the device, L2 flushed before each step,
    CUDA events around the two kernels.  Bytes: every cache row the step
    reads once (for top-k the gathered rows and the indices) + Q + O + LSE."""
    import torch

    import flagattention_b200 as fa
    from flagattention_b200 import _torch as fat
    from flagattention_b200.mla import MlaCall

    spec = OTHER[args.config]
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lens = other_lens(args.config)
    if args.batch:
        lens = lens[:args.batch]
    B, s_q, topk = len(lens), spec["s_q"], spec["topk"]
    g = torch.Generator(device=dev).manual_seed(SEED + args.config)
    pages_per = (lens + PAGE - 1) // PAGE
    npages = int(pages_per.sum())
    kcache = torch.empty((npages, PAGE, 1, D_QK), dtype=torch.bfloat16, device=dev)
    for lo in range(0, npages, 8192):
        hi = min(npages, lo + 8192)
        kcache[lo:hi] = torch.randn((hi - lo, PAGE, 1, D_QK), generator=g, device=dev)
    q = torch.randn((B, s_q, H_Q, D_QK), generator=g, device=dev, dtype=torch.bfloat16)
    perm = np.random.RandomState(SEED + 100 + args.config).permutation(npages).astype(np.int32)
    bt_np = np.zeros((B, int(pages_per.max())), np.int32)
    off = 0
    for i, k in enumerate(pages_per):
        bt_np[i, :k] = perm[off:off + k]
        off += k
    bt = torch.from_numpy(bt_np).to(dev)
    seq = torch.from_numpy(lens).to(dev)
    idx = None
    if topk:
        rs = np.random.RandomState(SEED + 200)
        idx_np = np.full((B, s_q, topk), -1, np.int32)
        for b, n in enumerate(lens):
            k = min(int(n), topk)
            pos = np.sort(rs.choice(int(n), size=k, replace=False))
            idx_np[b, 0, :k] = bt_np[b][pos // PAGE] * PAGE + pos % PAGE
        idx = torch.from_numpy(idx_np).to(dev)
    meta, splits = fa.get_mla_metadata(seq, s_q * H_Q, 1, num_heads_q=H_Q if topk else None,
                                       topk=topk or None)
    out = torch.empty((B, s_q, H_Q, D_V), dtype=torch.bfloat16, device=dev)
    lse = torch.empty((B, H_Q, s_q), dtype=torch.float32, device=dev)
    call = MlaCall(q, kcache, kcache.stride(0), kcache.stride(1), npages, PAGE, bt, seq, 0, meta,
                   splits, out, lse, D_QK ** -0.5, causal=spec["causal"], indices=idx)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step(ev):
        flush.fill_(1)
        ev[0].record(stream)
        call.partial()
        ev[1].record(stream)
        call.combine()
        ev[2].record(stream)

    for _ in range(args.warmup):
        step([torch.cuda.Event(enable_timing=True) for _ in range(3)])
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    for i in range(args.steps):
        step(evs[i])
    torch.cuda.synchronize()
    assert fat.read_status(dev) == 0, "device wait timeout in the timed region"
    dec_ms = sum(e[0].elapsed_time(e[1]) for e in evs) / args.steps
    step_ms = dec_ms + sum(e[1].elapsed_time(e[2]) for e in evs) / args.steps
    rows = int(np.minimum(lens, topk).sum()) if topk else int(lens.astype(np.int64).sum())
    qo = B * s_q * H_Q * (D_QK * 2 + D_V * 2 + 4)
    nbytes = rows * D_QK * 2 + qo + (B * s_q * topk * 4 if topk else 0)
    flops = rows * 2 * s_q * H_Q * (D_QK + D_V)
    peak_gbs, peak_tf, peak_kind = measured_peaks()
    tokens = B * s_q
    line = {"metric": METRIC, "value": tokens / (step_ms * 1e-3), "unit": "tok/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) bf16)",
            "config": {"workload": spec["workload"], "baseline_config": args.config,
                       "batch": B, "seq_q": s_q, "heads_q": H_Q, "topk": topk,
                       "causal": spec["causal"], "page_size": PAGE,
                       "l2": "flushed before every step (256 MB write, outside the events)"},
            "ms_decode_kernel": dec_ms, "ms_combine_kernel": step_ms - dec_ms,
            "roofline": {"bound": "hbm", "achieved": nbytes / (dec_ms * 1e-3) / 1e9,
                         "peak": peak_gbs, "unit": "GB/s",
                         "frac": nbytes / (dec_ms * 1e-3) / 1e9 / peak_gbs,
                         "peak_source": peak_kind, "algorithmic_bytes_per_launch": nbytes},
            "tensor_tflops_decode": flops / (dec_ms * 1e-3) / 1e12,
            "tensor_frac_decode": flops / (dec_ms * 1e-3) / 1e12 / peak_tf,
            "gpu_launches": 2 * args.steps}
    print(json.dumps(line))


def run_gqa_only(args):
    """`--gqa`: the grouped-query record alone, one GPU, one JSON line."""
    import torch

    c = gqa_shape(args.gqa)
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)   # > 126 MB L2
    rec = run_gqa(args, dev, flush, c)
    rec["warmup"] = args.warmup
    print(json.dumps(rec), flush=True)


def main():
    args = parse()
    if args.gqa is not None:
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable":
                              "the reference arm is timed on the headline config only"}))
        else:
            run_gqa_only(args)
    elif args.config != 2:
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable":
                              "the reference arm is timed on the headline config only"}))
        else:
            run_other(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
