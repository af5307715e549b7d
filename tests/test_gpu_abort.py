"""The MLA decode's abort path: bounded waits, unwinding, and the teardown
drain of P transfers in flight.

Runs the test build of the library (libflagattn_b200_aborttest.so, compiled
with FA_DEBUG_ABORT_TEST: waits give up after about 10 ms, and the value
CTA's metadata-read arrival for P block 6 is never made) in a child process.
The PV issuer's wait for that arrival runs out while the score CTA has
blocks 7-9 in flight, so every role unwinds and the teardown must account
for the blocks sent but not consumed.  The child checks that the decode
returns with a time-out status and that the same CUDA context then runs a
grouped-query decode correctly.  No fault or hang is involved: a lost
arrival is a wait that nothing completes.
"""

import json
import os
import subprocess
import sys

import pytest

from flagattention_b200 import build

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import json, os, sys
sys.path.insert(0, os.environ["FA_ROOT"])
import torch
import flagattention_b200 as fa
from flagattention_b200 import _lib, _torch as fat

assert os.path.basename(_lib.LIB_PATH) == "libflagattn_b200_aborttest.so"
dev = torch.device("cuda", 0)
g = torch.Generator(device=dev).manual_seed(3)
B, H, ctx = 4, 128, 2048
pages = B * ctx // 64
kc = torch.randn((pages, 64, 1, 576), generator=g, device=dev).to(torch.bfloat16)
bt = torch.randperm(pages, generator=g, device=dev).to(torch.int32).view(B, -1)
lens = torch.full((B,), ctx, dtype=torch.int32, device=dev)
q = torch.randn((B, 1, H, 576), generator=g, device=dev).to(torch.bfloat16)
# two parts of 64 blocks each: every cluster reaches P block 6
meta, splits = fa.get_mla_metadata(lens, H, 1, num_sm_parts_override=2)
fa.flash_mla_with_kvcache(q, kc, bt, lens, 512, meta, splits)
torch.cuda.synchronize()
status = fat.read_status(dev)

# the context still works: a grouped-query paged decode against torch
qq = torch.randn((2, 16, 128), generator=g, device=dev).to(torch.bfloat16)
kk = torch.randn((8, 2, 16, 128), generator=g, device=dev).to(torch.bfloat16)
vv = torch.randn((8, 2, 16, 128), generator=g, device=dev).to(torch.bfloat16)
bt2 = torch.arange(8, dtype=torch.int32, device=dev).view(2, 4)
l2 = torch.tensor([64, 50], dtype=torch.int32, device=dev)
o2 = fa.paged_attention(qq, kk, vv, l2, bt2, 128 ** -0.5, 64)
torch.cuda.synchronize()
err = 0.0
for s in range(2):
    n = int(l2[s])
    k = kk[bt2[s]].permute(1, 0, 2, 3).reshape(2, -1, 128)[:, :n].float()
    v = vv[bt2[s]].permute(1, 0, 2, 3).reshape(2, -1, 128)[:, :n].float()
    qh = qq[s].float().view(2, 8, 128)
    p = torch.softmax(qh @ k.transpose(1, 2) * 128 ** -0.5, dim=-1)
    ref = (p @ v).reshape(16, 128)
    err = max(err, (o2[s].float() - ref).abs().max().item())
print(json.dumps({"status": status, "gqa_err": err, "gqa_status": fat.read_status(dev)}))
"""


def test_decode_unwinds_after_lost_arrival():
    # built next to the shipped library by build() (__graft_entry__.build)
    assert os.path.exists(build.ABORT_TEST_LIB), "build the library first"
    env = dict(os.environ, FA_LIB_PATH=build.ABORT_TEST_LIB, FA_ROOT=ROOT)
    r = subprocess.run([sys.executable, "-c", CHILD], env=env, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    res = json.loads(r.stdout.strip().splitlines()[-1])
    # a wait ran out: a producer (1), the PV issuer (2) or the softmax /
    # epilogue side (3) -- the roles give up within the same ~10 ms and the
    # last writer of the status word wins.  The drain waits run last, so a
    # drain time-out (5), meaning a sent block never landed, would show.
    assert res["status"] in (1, 2, 3), res
    assert res["gqa_status"] == 0 and res["gqa_err"] < 2e-2, res
