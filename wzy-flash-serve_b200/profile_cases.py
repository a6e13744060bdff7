"""Small cases of single kernels for ncu captures (one kernel, a few launches, < 3 GB on the device).

    python wzy-flash-serve_b200/profile_cases.py <case> [reps]

cases: conv (PLE causal conv), fp8 (fp8 PLE gather, 2 GB table), kv (k RoPE + INT8 KV append),
grnorm / grq8 (4-stream norm, plain / with Q8_0), gate (PLE gate), hcmix (stream mixing),
grwrite (gated residual write), quant (int8 activation quantisation). 4096 tokens, n_embd 2560.
"""
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import wzyb200 as wz  # noqa: E402

which = sys.argv[1]
reps = int(sys.argv[2]) if len(sys.argv) > 2 else 3
dev = "cuda:0"
torch.cuda.set_device(0)
wz.lib().wzyb_prepare_device()
g = torch.Generator(device=dev).manual_seed(1)
T, NE, HC = 4096, 2560, 4

if which == "conv":
    hcd = NE * HC
    norm = torch.randn((T, hcd), generator=g, device=dev)
    cw = torch.randn((hcd, 4), generator=g, device=dev)
    hist = torch.randn((hcd, 9), generator=g, device=dev)
    gv = torch.randn((T, hcd), generator=g, device=dev)
    R = torch.randn((T, hcd), generator=g, device=dev)
    fn = lambda: wz.ple_conv_f32(norm, cw, hist, gv, R, T, hcd)  # noqa: E731
elif which == "fp8":
    vocab = [800011 + 2 * i for i in range(16)]
    hsh = wz.ple_fp8_hash(vocab=vocab)
    rows = sum(vocab)
    table = torch.randint(0, 256, (rows, 160), generator=g, device=dev, dtype=torch.uint8)
    ids = torch.randint(0, 248320, (T,), generator=g, device=dev, dtype=torch.int32)
    out = torch.empty((T, 2560), device=dev)
    fn = lambda: wz.ple_gather_fp8_f32(table, 160, 0.5, hsh, ids, out)  # noqa: E731
elif which == "kv":
    k = torch.randn((T, 512), generator=g, device=dev).half()
    v = torch.randn((T, 512), generator=g, device=dev).half()
    kg = (0.02 * torch.randn(256, generator=g, device=dev)).half()
    pl = [torch.zeros((T, 512), dtype=torch.int8, device=dev) if i % 2 == 0 else
          torch.zeros((T, 8), dtype=torch.int16, device=dev) for i in range(8)]
    cache = wz.kv_cache(*pl[:4], T, T, *pl[4:])
    c = torch.empty((T, 32), device=dev)
    s = torch.empty((T, 32), device=dev)
    wz.rope_table(c, s, T, 64, 1e7)
    fn = lambda: wz.k_rope_kv_append(k, kg, v, c, s, T, 2, 256, cache, rot_dims=64, w_offset=1.0)  # noqa: E731
elif which in ("grnorm", "grq8", "gate", "hcmix", "grwrite", "quant"):
    R = torch.randn((T * HC, NE), generator=g, device=dev)
    blk = torch.randn((T, NE), generator=g, device=dev)
    inj = torch.randn((T * HC,), generator=g, device=dev)
    wn = 1 + 0.02 * torch.randn((HC, NE), generator=g, device=dev)
    xn = torch.empty((T * HC, NE), device=dev)
    xq = torch.empty((T * HC, NE), dtype=torch.int8, device=dev)
    xs = torch.empty((T * HC, NE // 32), device=dev)
    if which == "grnorm":
        fn = lambda: wz.gr_norm_f32(R, wn, blk, inj, xn, T, NE, HC)  # noqa: E731
    elif which == "grq8":
        fn = lambda: wz.gr_norm_q8_f32(R, wn, blk, inj, xn, xq, xs, T, NE, HC)  # noqa: E731
    elif which == "gate":
        q = torch.randn((T * HC, NE), generator=g, device=dev)
        fn = lambda: wz.ple_gate_f32(R, q, blk, xn, T, NE, HC)  # noqa: E731
    elif which == "hcmix":
        x16 = torch.randn((T, HC, NE), generator=g, device=dev).half()
        g16 = torch.randn((T, HC, NE), generator=g, device=dev).half()
        m16 = torch.empty((T, NE), dtype=torch.float16, device=dev)
        fn = lambda: wz.hc_mix(x16, g16, blk, m16, T, NE, HC)  # noqa: E731
    elif which == "grwrite":
        fn = lambda: wz.gr_write_f32(R, blk, inj, T, NE, HC)  # noqa: E731
    else:
        q16 = torch.empty((T * HC, NE), dtype=torch.int8, device=dev)
        s16 = torch.empty((T * HC, NE // 16), device=dev)
        fn = lambda: wz.quant_act_f32(R, xq, xs, q16, s16, T * HC, NE)  # noqa: E731
else:
    raise SystemExit(f"unknown case {which}")

for _ in range(reps):
    fn()
torch.cuda.synchronize()
print("ok", which)
