"""Multi-GPU tests (NCCL, one process per GPU; skipped with fewer than 2 GPUs).

- vocab-sharded sampling: each rank holds one column shard; candidate lists are
  all-gathered and merged on every rank; the result must equal the oracle's on
  the full rows, on every rank, tie rows included. Run twice: through
  torch.distributed (mxs_sampler.dist) and through the C ABI's one-call
  mxs_sample_vocabsharded over an NCCL communicator;
- row-sharded bench: bench.py under torchrun prints one JSON line."""
import json
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


WORKER = r'''
import os, sys, json, numpy as np, torch, torch.distributed as dist
sys.path.insert(0, os.path.join(os.environ["ROOT"], "minxfmr.cpp_b200"))
sys.path.insert(0, os.path.join(os.environ["ROOT"], "tests"))
rank = int(os.environ["RANK"]); world = int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
import workloads, oracle_lib
from mxs_sampler.dist import VocabShardedSampler
rows, V, k, T = 64, 151936, 50, 0.8
x = workloads.normal(77, rows, V, 2.0)
x[3, 1000:1040] = 9.5           # tie row inside one shard
x[5, [10, V - 10]] = 11.0       # tie across shards
u = oracle_lib.uniforms(77, rows)
cols = V // world
shard = torch.from_numpy(x[:, rank * cols:(rank + 1) * cols].copy()).cuda()
vs = VocabShardedSampler(V)
nxt, idx, prob, fl = vs.sample(shard, T, k, torch.from_numpy(u).cuda())
torch.cuda.synchronize()
n0, i0, p0 = oracle_lib.oracle_sample(x, T, k, u)
ok = bool((nxt.cpu().numpy() == n0).all() and (idx.cpu().numpy() == i0).all()
          and np.allclose(prob.cpu().numpy(), p0, rtol=1e-6, atol=0))
# the same through the C ABI: one mxs_sample_vocabsharded call per rank over an NCCL communicator
import mxs_sampler
from mxs_sampler import nccl
obj = [nccl.get_unique_id() if rank == 0 else None]
dist.broadcast_object_list(obj, 0)
comm = nccl.comm_init_rank(world, obj[0], rank)
ok_abi = True
whole = []
bf16 = torch.from_numpy(workloads.normal(78, 48, V, 2.0)).bfloat16().float().numpy()
for xx, kk in ((x, k), (bf16, k), (bf16, 8), (bf16, 128)):
    uu = oracle_lib.uniforms(78, xx.shape[0])
    sh = torch.from_numpy(xx[:, rank * cols:(rank + 1) * cols].copy()).cuda()
    n2, i2, p2, f2 = mxs_sampler.sample_vocabsharded(sh, T, kk, torch.from_numpy(uu).cuda(), comm)
    torch.cuda.synchronize()
    whole.append(mxs_sampler.vocabsharded_stats()[1])
    m0, j0, q0 = oracle_lib.oracle_sample(xx, T, kk, uu)
    ok_abi = ok_abi and bool((n2.cpu().numpy() == m0).all() and (i2.cpu().numpy() == j0).all()
                             and np.allclose(p2.cpu().numpy(), q0, rtol=1e-6, atol=0))
nccl.comm_destroy(comm)
print(json.dumps({"rank": rank, "ok": ok, "ok_abi": ok_abi, "exact_rows": int((fl.cpu().numpy() & 1).sum()),
                  "rows_gathered_whole": whole}), flush=True)
dist.destroy_process_group()
sys.exit(0 if (ok and ok_abi) else 3)
'''


def _need_gpus(n):
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


@pytest.mark.parametrize("world", [2, 4, 8])
def test_vocab_sharded_nccl(world):
    """The north-star split at world 8: 8 shards of 18,992 columns."""
    _need_gpus(world)
    port = _free_port()
    env = dict(os.environ, ROOT=ROOT, MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world),
               NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, "-c", WORKER], env=dict(env, RANK=str(r), LOCAL_RANK=str(r)),
                              stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True) for r in range(world)]
    outs = [p.communicate(timeout=600)[0] for p in procs]
    for p, o in zip(procs, outs):
        assert p.returncode == 0, o[-3000:]
        line = [l for l in o.splitlines() if l.startswith("{")][-1]
        d = json.loads(line)
        assert d["ok"] and d["ok_abi"]
        assert d["rows_gathered_whole"] == [0, 0, 0, 0], d  # ties resolved from lists, bf16 rows included


def test_bench_two_gpus_row_and_vocab_sharded():
    """bench.py under torchrun: the row-sharded line with per-rank times, and
    the vocab-sharded sub-record with zero parity mismatches."""
    _need_gpus(2)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", str(_free_port()), os.path.join(ROOT, "bench.py"), "--gpus", "2", "--steps",
           "20", "--warmup", "3", "--no-e2e"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=900, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-3000:]
    line = json.loads([l for l in r.stdout.splitlines() if l.startswith("{")][-1])
    assert line["n_gpus"] == 2 and line["value"] > 0 and line["cpu_baseline"] is None
    assert len(line["per_rank"]) == 2
    vs = line["vocab_sharded"]
    assert vs["shards"] == 2 and vs["parity_mismatch_rows"] == 0 and vs["value"] > 0


THREADS = r'''
import os, sys, json, threading, numpy as np, torch
sys.path.insert(0, os.path.join(os.environ["ROOT"], "minxfmr.cpp_b200"))
sys.path.insert(0, os.path.join(os.environ["ROOT"], "tests"))
import workloads, oracle_lib, mxs_sampler
from mxs_sampler import nccl
world = 2
rows, V, k, T = 32, 151936, 50, 0.8
x = workloads.normal(91, rows, V, 2.0)
x[3, 500:540] = 9.5  # a tie row: the list pass runs with both threads inside collectives
u = oracle_lib.uniforms(91, rows)
cols = V // world
comms = nccl.comm_init_all(list(range(world)))
out = [None] * world
def rank_thread(r):
    torch.cuda.set_device(r)
    sh = torch.from_numpy(x[:, r * cols:(r + 1) * cols].copy()).cuda()
    for _ in range(3):
        n, i, p, f = mxs_sampler.sample_vocabsharded(sh, T, k, torch.from_numpy(u).cuda(), comms[r])
    torch.cuda.synchronize()
    out[r] = (n.cpu().numpy(), i.cpu().numpy())
ts = [threading.Thread(target=rank_thread, args=(r,)) for r in range(world)]
[t.start() for t in ts]
[t.join() for t in ts]
n0, i0, _ = oracle_lib.oracle_sample(x, T, k, u)
ok = all(o is not None and (o[0] == n0).all() and (o[1] == i0).all() for o in out)
for c in comms:
    nccl.comm_destroy(c)
print(json.dumps({"ok": bool(ok)}))
sys.exit(0 if ok else 3)
'''


def test_vocab_sharded_one_thread_per_gpu():
    """Two ranks driven by two threads of one process, each with its own
    communicator (ncclCommInitAll): each call holds only its own device's lock
    across its collectives, so the ranks never wait on each other's lock."""
    _need_gpus(2)
    env = dict(os.environ, ROOT=ROOT, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-c", THREADS], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, (r.stdout + r.stderr)[-3000:]
    assert json.loads([l for l in r.stdout.splitlines() if l.startswith("{")][-1])["ok"]
