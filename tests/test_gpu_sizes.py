"""GPU edge sizes: empty calls, and calls whose element counts exceed 2^31 (64-bit index arithmetic).

Empty calls (T = 0 or n = 0) with real device buffers must return 0, launch nothing and leave every
buffer unchanged. The large cases build ~4 GB tensors on the device and check sampled rows -- the
first, the middle, the last and random ones -- against the CPU oracle with the parity tolerances of
test_gpu_kernels.py (bit-exact for the gather and the residual, 2 fp16 ulp for norms, RoPE and SwiGLU).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import ULP_TOL, assert_f16_close

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
EPS = 1e-6


def _sample_rows(T, seed, k=11):
    r = np.random.default_rng(seed)
    idx = {0, 1, T // 2, T - 2, T - 1} | set(r.integers(0, T, k).tolist())
    return np.array(sorted(idx), dtype=np.int64)


def _h(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def test_empty_calls_are_noops(wz):
    torch.cuda.set_device(0)
    f16, f32 = torch.float16, torch.float32
    x = torch.full((8, 2048), 1.5, dtype=f16, device=DEV)
    res = torch.full((8, 2048), -0.5, dtype=f16, device=DEV)
    w = torch.zeros(2048, dtype=f16, device=DEV)
    y = torch.full((8, 2048), 7.0, dtype=f16, device=DEV)
    R = torch.full((16, 2560), 2.0, dtype=f32, device=DEV)
    bo = torch.ones((4, 2560), dtype=f32, device=DEV)
    inj = torch.zeros(16, dtype=f32, device=DEV)
    wn = torch.ones((4, 2560), dtype=f32, device=DEV)
    xn = torch.full((16, 2560), 9.0, dtype=f32, device=DEV)
    q8 = torch.full((16, 2560), 3, dtype=torch.int8, device=DEV)
    s8 = torch.full((16, 80), 4.0, dtype=f32, device=DEV)
    hist = torch.full((10240, 9), 5.0, dtype=f32, device=DEV)
    conv_in = torch.ones((4, 10240), dtype=f32, device=DEV)
    cw = torch.ones((10240, 4), dtype=f32, device=DEV)
    ids = torch.zeros(8, dtype=torch.int32, device=DEV)
    table = torch.ones((16, 2048), dtype=f16, device=DEV)
    bufs = [x, res, w, y, R, bo, inj, wn, xn, q8, s8, hist, conv_in, cw, ids, table]
    before = [b.clone() for b in bufs]
    s = wz._stream()
    p = wz._ptr
    lib = wz.lib()
    assert lib.wzyb_add_rmsnorm_f16(p(x), p(res), p(w), p(y), 0, 2048, EPS, 1.0, s) == 0
    assert lib.wzyb_swiglu_f16(p(x), p(res), p(y), 0, s) == 0
    assert lib.wzyb_gdn_gated_norm_f16(p(x), p(res), p(w), p(y), 0, 16, 128, EPS, 0.0, wz.GATE_SIGMOID, s) == 0
    assert lib.wzyb_gr_norm_q8_f32(p(R), p(wn), p(bo), p(inj), p(xn), p(q8), p(s8), 0, 2560, 4, EPS, s) == 0
    assert lib.wzyb_gr_write_f32(p(R), p(bo), p(inj), 0, 2560, 4, s) == 0
    assert lib.wzyb_quant_act_f32(p(R), p(q8), p(s8), None, None, 0, 2560, s) == 0
    assert lib.wzyb_ple_conv_f32(p(conv_in), p(cw), p(hist), p(conv_in), p(R), 0, 10240, None, s) == 0
    assert lib.wzyb_embed_gather_f16(p(table), 16, 2048, p(ids), 0, p(y), wz.OOB_CLAMP, None, s) == 0
    c = torch.ones((8, 32), dtype=f32, device=DEV)
    wz.head_norm_rope(x, w, c, c, 0, 8, 256, 256, 2048, 64, EPS, 1.0)
    for b, b0 in zip(bufs, before):
        assert torch.equal(b, b0)
    assert wz.read_faults() == 0


def test_add_rmsnorm_beyond_int32(wz, orc):
    torch.cuda.set_device(0)
    n = 2048
    T = (1 << 31) // n + 3  # T * n > 2^31
    g = torch.Generator(device=DEV).manual_seed(71)
    x = torch.randn((T, n), generator=g, device=DEV, dtype=torch.float16)
    res = torch.randn((T, n), generator=g, device=DEV, dtype=torch.float16)
    w = (0.02 * torch.randn(n, generator=g, device=DEV)).half()
    idx = _sample_rows(T, 1)
    ti = torch.from_numpy(idx).to(DEV)
    x_s, res_s = _h(x[ti]), _h(res[ti])
    y = torch.empty_like(x)
    wz.add_rmsnorm_f16(x, res, w, y, EPS, 1.0)
    y_ref, res_ref = orc.add_rmsnorm_f16(x_s, res_s, _h(w), EPS, 1.0)
    assert np.array_equal(_h(res[ti]), res_ref)
    assert_f16_close(_h(y[ti]), y_ref, ULP_TOL, "add_rmsnorm rows past 2^31 elements")
    del x, res, y


def test_swiglu_beyond_int32(wz, orc):
    torch.cuda.set_device(0)
    n = (1 << 31) + 64
    g = torch.Generator(device=DEV).manual_seed(72)
    gate = torch.randn(n, generator=g, device=DEV, dtype=torch.float16)
    up = torch.randn(n, generator=g, device=DEV, dtype=torch.float16)
    out = torch.empty_like(gate)
    wz.swiglu(gate, up, out)
    for lo in (0, (1 << 31) - 4096, n - 8192):
        sl = slice(lo, lo + 8192)
        assert_f16_close(_h(out[sl]), orc.swiglu(_h(gate[sl]), _h(up[sl])), ULP_TOL, f"swiglu at {lo}")
    del gate, up, out


def test_qk_norm_rope_beyond_int32(wz, orc):
    torch.cuda.set_device(0)
    hd, rot = 256, 64
    T = (1 << 31) // (16 * hd) + 5  # q alone holds more than 2^31 elements
    g = torch.Generator(device=DEV).manual_seed(73)
    q = torch.randn((T, 16, hd), generator=g, device=DEV, dtype=torch.float16)
    k = torch.randn((T, 2, hd), generator=g, device=DEV, dtype=torch.float16)
    gq = (0.02 * torch.randn(hd, generator=g, device=DEV)).half()
    gk = (0.02 * torch.randn(hd, generator=g, device=DEV)).half()
    c, s = orc.rope_table(T, rot, 1e7)
    dc, ds = torch.from_numpy(c).to(DEV), torch.from_numpy(s).to(DEV)
    idx = _sample_rows(T, 3)
    ti = torch.from_numpy(idx).to(DEV)
    q_s, k_s = _h(q[ti]), _h(k[ti])
    wz.qk_norm_rope_f16(wz.head_tensor(q, gq, 16, hd, 16 * hd), wz.head_tensor(k, gk, 2, hd, 2 * hd), dc, ds, T, hd,
                        rot, EPS, 1.0)
    q_out, k_out = _h(q[ti]), _h(k[ti])
    for j, t in enumerate(idx):
        qr = orc.head_norm_rope(q_s[j].reshape(-1), _h(gq), c, s, 1, 16, hd, hd, 16 * hd, rot, EPS, 1.0, int(t))
        kr = orc.head_norm_rope(k_s[j].reshape(-1), _h(gk), c, s, 1, 2, hd, hd, 2 * hd, rot, EPS, 1.0, int(t))
        assert_f16_close(q_out[j].reshape(-1), qr, ULP_TOL, f"q token {t}")
        assert_f16_close(k_out[j].reshape(-1), kr, ULP_TOL, f"k token {t}")
    assert wz.read_faults() == 0
    del q, k


def test_gdn_gated_norm_beyond_int32(wz, orc):
    torch.cuda.set_device(0)
    H, hd = 32, 128
    T = (1 << 31) // (H * hd) + 7
    g = torch.Generator(device=DEV).manual_seed(74)
    o = torch.randn((T, H, hd), generator=g, device=DEV, dtype=torch.float16)
    z = torch.randn((T, H, hd), generator=g, device=DEV, dtype=torch.float16)
    gm = (1 + 0.02 * torch.randn(hd, generator=g, device=DEV)).half()
    y = torch.empty_like(o)
    wz.gdn_gated_norm(o, z, gm, y, T, H, hd, EPS, 0.0, wz.GATE_SIGMOID)
    idx = _sample_rows(T, 4)
    ti = torch.from_numpy(idx).to(DEV)
    want = orc.gdn_gated_norm(_h(o[ti]), _h(z[ti]), _h(gm), idx.size, H, hd, EPS, 0.0, 0)
    assert_f16_close(_h(y[ti]), want, ULP_TOL, "gdn rows past 2^31 elements")
    del o, z, y


def test_embed_gather_beyond_int32(wz):
    torch.cuda.set_device(0)
    vocab, n = 151936, 2048
    T = (1 << 31) // n + 9
    g = torch.Generator(device=DEV).manual_seed(75)
    table = (0.02 * torch.randn((vocab, n), generator=g, device=DEV)).half()
    ids = torch.randint(0, vocab, (T,), generator=g, device=DEV, dtype=torch.int32)
    out = torch.empty((T, n), dtype=torch.float16, device=DEV)
    wz.embed_gather_f16(table, ids, out)
    idx = _sample_rows(T, 5)
    ti = torch.from_numpy(idx).to(DEV)
    want = table[ids[ti].long()]
    assert torch.equal(out[ti].view(torch.int16), want.view(torch.int16))
    del table, out
