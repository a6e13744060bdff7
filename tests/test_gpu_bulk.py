"""GPU parity of the bulk (TMA) design of the gathers: rows copied global -> shared -> global by
cp.async.bulk, a ring of slots per warp (wzyb_set_kernel_variant(WZYB_FAM_GATHER, WZYB_VARIANT_RING)).

Bit-exact against the oracle for the token-embedding rows (any 16-byte multiple up to 16 KiB, both
out-of-range policies with the count), the PLE rows (head counts 1..32, head sizes 32..512 bytes, both
hash readings, history and EOS cuts) and the one-launch bundle of both; sizes cover a warp with fewer
units than slots, a warp that refills its ring many times, and more than 32 units per warp (the ids
are fetched 32 units at a time).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(autouse=True)
def _bulk(wz):
    torch.cuda.set_device(0)
    wz.read_faults(clear=True)
    wz.set_kernel_variant(wz.FAM_GATHER, wz.VARIANT_RING)
    yield
    torch.cuda.synchronize()
    wz.set_kernel_variant(wz.FAM_GATHER, wz.VARIANT_AUTO)
    assert wz.read_faults() == 0


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.mark.parametrize("T,row_bytes,policy", [(1, 4096, 0), (5, 16, 1), (777, 48, 0), (4096, 4096, 0),
                                                (4096, 16384, 1), (70001, 4096, 1), (3000, 272, 0)])
def test_bulk_embed_rows(wz, orc, T, row_bytes, policy):
    r = np.random.default_rng(T + row_bytes)
    vocab = 9001
    table = r.integers(0, 256, (vocab, row_bytes), dtype=np.uint8)
    ids = r.integers(-3, vocab + 3, T).astype(np.int32)
    out = torch.empty((T, row_bytes), dtype=torch.uint8, device=DEV)
    cnt = torch.zeros(1, dtype=torch.int32, device=DEV)
    wz.embed_gather_rows(dev(table), dev(ids), out, policy, cnt)
    want, bad = orc.embed_gather_rows(table, ids, policy)
    assert np.array_equal(host(out), want)
    assert int(host(cnt)[0]) == bad


@pytest.mark.parametrize("T,heads,rows,hd,variant,prev", [(1, 16, 1 << 12, 128, 0, None), (2, 16, 4099, 128, 1, (5, 6)),
                                                          (4096, 16, 1 << 20, 128, 0, None),
                                                          (70001, 16, 4099, 128, 0, (248044, 3)),
                                                          (333, 1, 777, 16, 1, (-1, 9)), (999, 32, 513, 256, 0, (2, 2)),
                                                          (128, 5, 1000, 64, 1, None)])
def test_bulk_ple_rows(wz, orc, T, heads, rows, hd, variant, prev):
    r = np.random.default_rng(T * heads + hd)
    tabs = [(r.standard_normal((rows, hd)) * 0.02).astype(np.float16) for _ in range(heads)]
    ids = r.integers(0, 151936, T).astype(np.int32)
    if T > 8:
        ids[[0, T // 3, T - 2]] = [248044, -5, 248044]
    out = torch.empty((T, heads * hd), dtype=torch.float16, device=DEV)
    wz.ple_gather_f16([dev(t) for t in tabs], dev(ids), out, prev_ids=prev, hash_variant=variant)
    want = orc.ple_gather_f16(tabs, ids, prev, 248044, variant)
    assert np.array_equal(host(out).view(np.uint16), want.view(np.uint16))


@pytest.mark.parametrize("T", [1, 3, 4096, 20000])
def test_bulk_embed_ple_bundle(wz, orc, T):
    r = np.random.default_rng(31 + T)
    vocab, hidden, heads, rows, hd = 7000, 2048, 16, 4099, 128
    table = (r.standard_normal((vocab, hidden)) * 0.02).astype(np.float16)
    tabs = [(r.standard_normal((rows, hd)) * 0.02).astype(np.float16) for _ in range(heads)]
    ids = r.integers(-1, vocab + 1, T).astype(np.int32)
    emb = torch.empty((T, hidden), dtype=torch.float16, device=DEV)
    ple = torch.empty((T, heads * hd), dtype=torch.float16, device=DEV)
    cnt = torch.zeros(1, dtype=torch.int32, device=DEV)
    dtabs = [dev(t) for t in tabs]
    args = wz.embed_ple_args(dev(table), dtabs, dev(ids), emb, ple, prev_ids=(11, 12), oob_count=cnt)
    wz.embed_ple_f16(args, T)
    want_e, bad = orc.embed_gather_rows(table, ids, 0)
    assert np.array_equal(host(emb).view(np.uint16), want_e.view(np.uint16))
    assert int(host(cnt)[0]) == bad
    want_p = orc.ple_gather_f16(tabs, ids, (11, 12), 248044, 0)
    assert np.array_equal(host(ple).view(np.uint16), want_p.view(np.uint16))
