"""Generate the golden fixtures by running FlagAttention's own reference code.

Run in a container that has the reference source tree (its ``src`` directory
on ``FLAG_ATTN_SRC``); the GPU box never runs this script.  Every fixture is
produced by the unmodified reference functions:

* ``flag_attn.testing.paged_attention``  (testing/paged.py:18-65)
* ``flag_attn.testing.flash_attention``  (testing/flash.py:19-84)
* ``flag_attn.split_kv.num_splits_herustic`` (split_kv.py:247-276)
* the partition rule of ``flag_attn.paged.attention`` (paged.py:54-67),
  executed from the reference's own source lines (it is inline code in a
  function that otherwise launches a GPU kernel).

Usage:  FLAG_ATTN_SRC=<reference>/src python tests/golden/make_golden.py
"""

import inspect
import json
import os
import sys
import textwrap

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from inputs import digest, mla_inputs, paged_pool, round_bf16, sparse_indices  # noqa: E402

if not os.environ.get("FLAG_ATTN_SRC"):
    sys.exit("set FLAG_ATTN_SRC to the reference's src/ directory (the one holding flag_attn/)")
sys.path.insert(0, os.environ["FLAG_ATTN_SRC"])
import flag_attn  # noqa: E402
import flag_attn.paged  # noqa: E402
from flag_attn.split_kv import num_splits_herustic  # noqa: E402

torch.set_num_threads(os.cpu_count() or 1)
D_QK, D_V, PAGE = 576, 512, 64


def t(x):
    return torch.from_numpy(np.ascontiguousarray(x))


def gather(kc, bt_row, n):
    rows = kc.reshape(kc.shape[0], kc.shape[1], -1)
    tok = np.arange(n)
    return rows[bt_row[tok // PAGE], tok % PAGE]


def ref_mla_dense(q, kc, bt, lens, causal):
    """Reference flash_attention on the gathered pages of each sequence."""
    B, s_q, H, _ = q.shape
    out = np.zeros((B, s_q, H, D_V), np.float32)
    lse = np.zeros((B, H, s_q), np.float32)
    for b in range(B):
        rows = gather(kc, bt[b], int(lens[b]))
        k = t(rows)[None, None]
        qb = t(q[b]).permute(1, 0, 2)[None]
        o, L, _ = flag_attn.testing.flash_attention(
            qb, k, k[..., :D_V], causal, sm_scale=D_QK ** -0.5,
            return_log_normalizer=True, upcast=True)
        out[b] = o[0].permute(1, 0, 2).numpy()
        lse[b] = L[0].numpy()
    return out, lse


def fixture_config1():
    """B=4, s_q=1, 16 heads, ctx U[64,1024], fp32 N(0,1)."""
    seed = 1001
    lens = np.random.RandomState(seed + 7).randint(64, 1025, size=4).astype(np.int32)
    q, kc, bt = mla_inputs(seed, 4, 1, 16, lens, bf16=False)
    scale = D_QK ** -0.5
    # paged oracle with the MLA adapter: V = K (576 wide), keep the first 512.
    o_paged = flag_attn.testing.paged_attention(
        t(q[:, 0]), t(kc).permute(0, 2, 1, 3).contiguous(),
        t(kc).permute(0, 2, 1, 3).contiguous(), t(bt), t(lens), scale)[..., :D_V]
    out, lse = ref_mla_dense(q, kc, bt, lens, False)
    np.savez_compressed(
        os.path.join(HERE, "mla_config1.npz"), seed=seed, lens=lens, block_table=bt,
        digest=digest(q, kc), out_paged=o_paged.numpy()[:, None], out=out, lse=lse)


def fixture_mtp():
    seed = 2002
    lens = np.array([40, 70, 130], np.int32)
    q, kc, bt = mla_inputs(seed, 3, 2, 16, lens, bf16=True)
    out, lse = ref_mla_dense(q, kc, bt, lens, True)
    out_nc, lse_nc = ref_mla_dense(q, kc, bt, lens, False)
    np.savez_compressed(
        os.path.join(HERE, "mla_mtp_causal.npz"), seed=seed, lens=lens, block_table=bt,
        digest=digest(q, kc), out=out, lse=lse, out_noncausal=out_nc, lse_noncausal=lse_nc)


def fixture_sparse():
    seed = 3003
    lens = np.array([100, 700], np.int32)
    topk = 128
    q, kc, bt = mla_inputs(seed, 2, 2, 16, lens, bf16=True)
    idx = sparse_indices(seed + 5, lens, 2, topk, bt)
    rows_all = kc.reshape(-1, D_QK)
    out = np.zeros((2, 2, 16, D_V), np.float32)
    lse = np.zeros((2, 16, 2), np.float32)
    for b in range(2):
        for i in range(2):
            sel = idx[b, i][idx[b, i] >= 0]
            k = t(rows_all[sel])[None, None]
            o, L, _ = flag_attn.testing.flash_attention(
                t(q[b, i])[None, :, None, :], k, k[..., :D_V], False,
                sm_scale=D_QK ** -0.5, return_log_normalizer=True, upcast=True)
            out[b, i] = o[0, :, 0].numpy()
            lse[b, :, i] = L[0, :, 0].numpy()
    np.savez_compressed(
        os.path.join(HERE, "mla_sparse.npz"), seed=seed, lens=lens, block_table=bt,
        topk=topk, indices=idx, digest=digest(q, kc), out=out, lse=lse)


def fixture_paged_gqa():
    """Small cases in the style of tests/flag_attn/test_paged_attention.py."""
    cases = [(2, 8, 1, 64, 16, 100), (3, 16, 8, 128, 16, 300),
             (1, 12, 1, 64, 16, 2), (2, 8, 4, 32, 128, 200)]
    store = {}
    for ci, (S, Hq, G, D, blk, max_len) in enumerate(cases):
        g = torch.Generator().manual_seed(4000 + ci)
        Hkv = Hq // G
        width = (max_len + blk - 1) // blk
        nblocks = width + 3
        scale = D ** -0.5
        lens = torch.randint(1, max_len, [S], generator=g, dtype=torch.int32) if max_len > 1 \
            else torch.ones(S, dtype=torch.int32)
        lens[0] = max_len
        q = (torch.rand(S, Hq, D, generator=g) * 2 - 1) * scale
        k = (torch.rand(nblocks, Hkv, blk, D, generator=g) * 2 - 1) * scale
        v = (torch.rand(nblocks, Hkv, blk, D, generator=g) * 2 - 1) * scale
        q, k, v = q.half(), k.half(), v.half()
        bt = torch.randint(0, nblocks, (S, width), generator=g, dtype=torch.int32)
        ref = flag_attn.testing.paged_attention(q, k, v, bt, lens, scale)
        ref32 = flag_attn.testing.paged_attention(q.float(), k.float(), v.float(), bt, lens, scale)
        for name, val in dict(q=q, k=k, v=v, bt=bt, lens=lens, out=ref, out_f32=ref32).items():
            store[f"c{ci}_{name}"] = val.numpy()
        store[f"c{ci}_scale"] = np.float32(scale)
    store["num_cases"] = len(cases)
    np.savez_compressed(os.path.join(HERE, "paged_gqa.npz"), **store)


def fixture_split_kv():
    """flash_attention reference (with LSE) on contiguous KV, decode-sized M."""
    cases = [(2, 4, 2, 1, 300, 64, False), (2, 4, 2, 2, 120, 128, True),
             (1, 2, 1, 4, 130, 32, True), (2, 4, 1, 1, 77, 16, False)]
    store = {}
    for ci, (B, Hq, Hk, M, N, D, causal) in enumerate(cases):
        g = torch.Generator().manual_seed(5000 + ci)
        q = (torch.randn(B, Hq, M, D, generator=g) * 2).half()
        k = (torch.randn(B, Hk, N, D, generator=g) * 2).half()
        v = (torch.randn(B, Hk, N, D, generator=g) * 2).half()
        o, L, _ = flag_attn.testing.flash_attention(q, k, v, causal, upcast=True,
                                                    return_log_normalizer=True)
        o32 = flag_attn.testing.flash_attention(q.float(), k.float(), v.float(), causal)
        for name, val in dict(q=q, k=k, v=v, out=o, out_f32=o32, lse=L).items():
            store[f"c{ci}_{name}"] = val.numpy()
        store[f"c{ci}_causal"] = np.int32(causal)
    store["num_cases"] = len(cases)
    np.savez_compressed(os.path.join(HERE, "split_kv.npz"), **store)


def fixture_combine():
    """Partials from the reference on KV sub-ranges + its full-range result."""
    g = torch.Generator().manual_seed(6000)
    B, H, M, N, D = 1, 4, 1, 256, 64
    q = torch.randn(B, H, M, D, generator=g)
    k = torch.randn(B, H, N, D, generator=g)
    v = torch.randn(B, H, N, D, generator=g)
    bounds = [0, 50, 51, 256]      # uneven, one single-token split
    po, pl = [], []
    for a, b in zip(bounds[:-1], bounds[1:]):
        o, L, _ = flag_attn.testing.flash_attention(q, k[:, :, a:b], v[:, :, a:b], False,
                                                    return_log_normalizer=True)
        po.append(o.numpy())
        pl.append(L.numpy())
    o, L, _ = flag_attn.testing.flash_attention(q, k, v, False, return_log_normalizer=True)
    np.savez_compressed(os.path.join(HERE, "combine.npz"), part_o=np.stack(po),
                        part_lse=np.stack(pl), out=o.numpy(), lse=L.numpy())


def _reference_paged_rule():
    """Wrap the reference's inline split rule (paged.py:54-67) as a function."""
    src = inspect.getsource(flag_attn.paged.attention).splitlines()
    start = next(i for i, s in enumerate(src) if s.strip() == "if num_splits == 0:")
    stop = next(i for i, s in enumerate(src) if "next_power_of_2(partition_size)" in s)
    body = textwrap.dedent("\n".join(src[start:stop + 1]))
    fn_src = ("def rule(num_seqs, num_kv_heads, max_context_len, kv_block_size, num_sms, num_splits):\n"
              "    partition_size = 0\n" + textwrap.indent(body, "    ") +
              "\n    return num_splits, partition_size\n")
    ns = {"triton": flag_attn.paged.triton}
    exec(fn_src, ns)
    return ns["rule"]


def fixture_heuristics():
    rule = _reference_paged_rule()
    paged = []
    for num_sms in (108, 132, 148):
        for seqs in (1, 4, 32, 64, 200, 400):
            for hkv in (1, 8):
                for ctx in (2, 512, 1024, 1025, 2048, 4095, 4096, 8192, 131072):
                    for blk in (16, 64, 128, 256, 512):
                        for req in (0, 1, 2, 3, 5, 8):
                            try:
                                ns, ps = rule(seqs, hkv, ctx, blk, num_sms, req)
                            except Exception:  # noqa: BLE001
                                continue
                            paged.append([seqs, hkv, ctx, blk, num_sms, req, int(ns), int(ps)])
    splitkv = []
    for num_sms in (108, 148):
        for B in (1, 2, 4):
            for H in (1, 2, 4, 16, 128):
                for M in (1, 2, 4, 16, 17):
                    for N in (1, 77, 612, 1034, 4001, 8202, 65536):
                        s = num_splits_herustic(B, H, M, N, 16, 128, num_sms, 128)
                        splitkv.append([B, H, M, N, 16, 128, num_sms, 128, int(s)])
    with open(os.path.join(HERE, "heuristics.json"), "w") as f:
        json.dump({"paged_rule": paged, "split_kv": splitkv}, f, separators=(",", ":"))


if __name__ == "__main__":
    fixture_heuristics()
    fixture_combine()
    fixture_split_kv()
    fixture_paged_gqa()
    fixture_sparse()
    fixture_mtp()
    fixture_config1()
    print("fixtures written to", HERE)
