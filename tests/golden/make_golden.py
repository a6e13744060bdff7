"""Generate tests/golden/ref_kernels_golden.npz: small seeded inputs run through the REFERENCE's own
kernels (oracle/_ref/libwzyref.so, built from the reference's unmodified headers) on a GPU, plus the
reference's host RoPE table builder at sampled positions. The CPU test suite checks the oracle
against these outputs (tests/test_golden_cpu.py), so the oracle stays pinned on machines without a
GPU or the reference sources.

Every device buffer handed to a kernel is kept in `keep` until after the synchronisation: a pointer
taken from a temporary tensor would let the caching allocator hand the same block to the next one.

Usage (on a machine with an sm_100 GPU and the built oracle/_ref library):
    python tests/golden/make_golden.py --out tests/golden/ref_kernels_golden.npz
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.join(ROOT, "tests", "golden", "ref_kernels_golden.npz"))
    args = ap.parse_args()

    import torch

    import oracle as orc

    ref = orc.ref_lib()
    dev = "cuda:0"
    s = torch.cuda.current_stream().cuda_stream
    r = np.random.default_rng(20261201)
    g = {}
    keep = []

    def D(a):
        t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        keep.append(t)
        return t.data_ptr()

    def H(t):
        torch.cuda.synchronize()
        return t.cpu().numpy()

    def out(shape, dtype):
        t = torch.empty(shape, dtype=dtype, device=dev)
        keep.append(t)
        return t

    # residual add + RMSNorm, single stream (pf_gr_norm_fp16, gate 1.0 via inj = 0)
    T, n = 16, 2048
    x = r.standard_normal((T, n)).astype(np.float16)
    res = r.standard_normal((T, n)).astype(np.float16)
    w = (0.02 * r.standard_normal(n)).astype(np.float16)
    dR = torch.from_numpy(res.astype(np.float32)).to(dev)
    dxn = out((T, n), torch.float16)
    assert ref.ref_pf_gr_norm_fp16(dR.data_ptr(), D((np.float32(1) + w.astype(np.float32)).astype(np.float32)),
                                   D(x.astype(np.float32)), D(np.zeros(T, np.float32)), dxn.data_ptr(), T, n, 1,
                                   1e-6, s) == 0
    g.update(addnorm_x=x, addnorm_res=res, addnorm_w=w, addnorm_y=H(dxn), addnorm_R=H(dR))

    # hyper-connection norm, 4 streams (fused_gr_norm_multi)
    T, n, hc = 4, 256, 4
    R = r.standard_normal((T * hc, n)).astype(np.float32)
    bo = r.standard_normal((T, n)).astype(np.float32)
    inj = r.standard_normal(T * hc).astype(np.float32)
    wn = (1 + 0.02 * r.standard_normal((hc, n))).astype(np.float32)
    dR = torch.from_numpy(R).to(dev)
    dxn = out((T * hc, n), torch.float32)
    assert ref.ref_fused_gr_norm_multi(dR.data_ptr(), D(wn), D(bo), D(inj), dxn.data_ptr(), T, n, hc, 1e-6, s) == 0
    g.update(hc_R=R, hc_bo=bo, hc_inj=inj, hc_w=wn, hc_xn=H(dxn), hc_Rout=H(dR))

    # per-head norm + RoPE (fused_head_norm_rope_multi), base position 1000
    T, heads, hd = 16, 4, 256
    q = r.standard_normal((T, heads, hd)).astype(np.float16)
    gq = (0.02 * r.standard_normal(hd)).astype(np.float16)
    c, sn = orc.ref_rope_table(1100, 1e7)
    dq = torch.from_numpy(q.astype(np.float32)).to(dev)
    assert ref.ref_fused_head_norm_rope_multi(dq.data_ptr(), D((np.float32(1) + gq.astype(np.float32))
                                                               .astype(np.float32)), D(c), D(sn),
                                              D(np.array([1000], np.int32)), T, heads, hd, hd, heads * hd, 1e-6,
                                              s) == 0
    g.update(rope_q=q, rope_gamma=gq, rope_out=H(dq))

    # GDN gated norm (pf_gdn_rmsnorm_gate_parallel)
    T, Hh, hd = 16, 8, 128
    o = r.standard_normal((T, Hh, hd)).astype(np.float16)
    z = r.standard_normal((T, Hh, hd)).astype(np.float16)
    gm = (1 + 0.02 * r.standard_normal(hd)).astype(np.float16)
    dy = out((T, Hh, hd), torch.float16)
    assert ref.ref_pf_gdn_rmsnorm_gate_parallel(D(o.astype(np.float32)), D(z.astype(np.float32)),
                                                D(gm.astype(np.float32)), dy.data_ptr(), T, Hh, 1e-6, s) == 0
    g.update(gdn_o=o, gdn_z=z, gdn_gamma=gm, gdn_y=H(dy))

    # SwiGLU (silu_mul_multi) and interleaved -> fp16 (pf_silu_mul_interleaved_to_fp16)
    gg = (3 * r.standard_normal(8192)).astype(np.float16)
    uu = r.standard_normal(8192).astype(np.float16)
    so = out(8192, torch.float32)
    assert ref.ref_silu_mul_multi(D(gg.astype(np.float32)), D(uu.astype(np.float32)), so.data_ptr(), 8192, s) == 0
    T, nff = 8, 640
    gu = (2 * r.standard_normal((T, 2 * nff))).astype(np.float32)
    o16 = out((T, nff), torch.float16)
    assert ref.ref_pf_silu_mul_interleaved_to_fp16(D(gu), o16.data_ptr(), T, nff, s) == 0
    g.update(swiglu_g=gg, swiglu_u=uu, swiglu_out=H(so), swil_gu=gu, swil_out=H(o16))

    # the reference's host RoPE table at sampled positions up to 262,143
    c, sn = orc.ref_rope_table(262144, 1e7)
    pos = np.array(list(range(64)) + [4095, 4096, 65535, 65536, 131071, 200000, 262143], dtype=np.int64)
    g.update(ropetab_pos=pos, ropetab_cos=c[pos], ropetab_sin=sn[pos])

    torch.cuda.synchronize()
    np.savez_compressed(args.out, **g)
    print(f"wrote {args.out} ({os.path.getsize(args.out)} bytes, {len(g)} arrays)")


if __name__ == "__main__":
    main()
