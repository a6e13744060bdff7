"""CPU, world_size 2 over gloo: the token-sharded path's host logic. Each rank takes its row range
from wzyb_shard_rows, its 2-id PLE history halo from wzyb_ple_halo and its RoPE position base from
its first row, runs its shard (on the oracle: no GPU here), and rank 0 checks that the gathered
shards equal the unsharded computation bit for bit. No data-path collective is involved; gloo only
gathers the results for the check."""
from __future__ import annotations

import json
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(T):
    r = np.random.default_rng(77)
    return {
        "q": r.standard_normal((T, 4, 256)).astype(np.float16),
        "gq": (0.02 * r.standard_normal(256)).astype(np.float16),
        "x": r.standard_normal((T, 512)).astype(np.float16),
        "res": r.standard_normal((T, 512)).astype(np.float16),
        "w": (0.02 * r.standard_normal(512)).astype(np.float16),
        "ids": r.integers(0, 151936, T).astype(np.int32),
        "tables": [(0.02 * r.standard_normal((4096, 64))).astype(np.float16) for _ in range(16)],
    }


def _shard_outputs(orc, wz, d, r0, n, T, seq_prev):
    c, s = orc.rope_table(T, 64, 1e7)
    q = orc.head_norm_rope(d["q"][r0:r0 + n].reshape(-1), d["gq"], c, s, n, 4, 256, 256, 1024, 64, 1e-6, 1.0,
                           base_pos=r0)
    y, res = orc.add_rmsnorm_f16(d["x"][r0:r0 + n], d["res"][r0:r0 + n], d["w"], 1e-6, 1.0)
    halo = wz.ple_halo(d["ids"], r0, seq_prev)
    ple = orc.ple_gather_f16(d["tables"], d["ids"][r0:r0 + n], halo, 248044, 0)
    return {"q": q.reshape(n, 4, 256), "y": y, "res": res, "ple": ple}


def _worker(rank, world, port, T, seq_prev, out_path):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "wzy-flash-serve_b200"), os.path.join(ROOT, "oracle")]
    import oracle as orc
    import wzyb200 as wz

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        orc.set_threads(1)
        d = _inputs(T)
        r0, n = wz.shard_rows(T, world, rank)
        mine = _shard_outputs(orc, wz, d, r0, n, T, seq_prev)
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        if rank == 0:
            full = _shard_outputs(orc, wz, d, 0, T, T, seq_prev)
            ok = {}
            for k in full:
                cat = np.concatenate([g[k] for g in gathered])
                ok[k] = bool(np.array_equal(cat.view(np.uint16), full[k].view(np.uint16)))
            with open(out_path, "w") as f:
                json.dump(ok, f)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("T,seq_prev", [(301, None), (64, (5, 248044))])
def test_two_rank_shards_equal_unsharded(tmp_path, T, seq_prev):
    out = str(tmp_path / "ok.json")
    mp.start_processes(_worker, args=(2, _free_port(), T, seq_prev, out), nprocs=2, start_method="spawn")
    with open(out) as f:
        ok = json.load(f)
    assert ok and all(ok.values()), ok


def test_reference_arm_under_torchrun_prints_once():
    """bench.py --impl reference launched as 2 ranks: rank 0 alone works and prints one JSON line."""
    env = dict(os.environ, OMP_NUM_THREADS="2")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", str(_free_port()), os.path.join(ROOT, "bench.py"), "--impl", "reference",
           "--gpus", "2", "--steps", "2", "--warmup", "1"]
    p = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, p.stdout
    rec = json.loads(lines[0])
    assert rec["impl"] == "reference" and rec["value"] > 0 and rec["cpu_baseline"]["kind"] == "port"
    assert rec["e2e"]["h2d_bytes_per_step"] == 0
