"""bench.py's accounting follows the library's own rules: which bundles run as one launch (the
per-bundle sizes in csrc/bundle.cu) and the algorithmic bytes per token of each op (the tensors the
entry points read and write once)."""
from __future__ import annotations

import os
import re

import bench
from conftest import ROOT

BUNDLE_CU = os.path.join(ROOT, "wzy-flash-serve_b200", "csrc", "bundle.cu")


def _lib_limits():
    src = open(BUNDLE_CU).read()
    out = {}
    for name, key in (("kFuseMaxAttn", "attn_b"), ("kFuseMaxAct", "act_b"), ("kFuseMaxGather", "gath_b")):
        m = re.search(r"constexpr double " + name + r" = ([0-9.]+) \* \(1 << (\d+)\);", src)
        assert m, name
        out[key] = float(m.group(1)) * (1 << int(m.group(2)))
    return out


def test_one_launch_sizes_match_the_library():
    assert _lib_limits() == bench.FUSE_MAX_BYTES


def test_bundle_rule_at_the_benchmark_shards():
    # 4096 tokens: every bundle is one launch; 262,144 tokens (1 GPU) and 32,768 (8 GPUs): the act
    # bundle is two launches; attn_prep stays one launch up to ~37K tokens
    assert all(bench.bundle_fused(b, 4096) for b in ("attn_b", "act_b", "gath_b"))
    assert not bench.bundle_fused("attn_b", 262144) and not bench.bundle_fused("act_b", 262144)
    assert bench.bundle_fused("attn_b", 32768) and not bench.bundle_fused("act_b", 32768)
    assert not bench.bundle_fused("gath_b", 8192)


def test_bytes_per_token():
    b = bench.BYTES_PER_TOKEN
    assert b["norm"] == 4 * 2048 * 2            # x, residual read; residual, y written (fp16)
    assert b["qk"] == 2 * 18 * 256 * 2          # 16 q + 2 k heads of 256, in place
    assert b["swi"] == 3 * 11 * 512 * 2         # gate, up, act over 11 expert rows of 512
    assert b["gdn"] == 3 * 32 * 128 * 2         # o, z, y
    # the configs[1] bundle: activations + the norm weight + the q and k gammas
    assert bench.bundle_bytes("attn_b", 4096) == 4096 * (b["norm"] + b["qk"]) + 2048 * 2 + 2 * 256 * 2
