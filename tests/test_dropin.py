"""The drop-in check: oracle/stage_dropin.cu puts the reference's executor headers (src/wzy_stage_v2.cuh,
src/wzy_mtp.cuh, src/wzy_prefill_tc.cuh) and include/wzyb200.h in one translation unit and makes every
launch-site replacement with the reference's own globals, members and pointer types.

CPU: the unit compiles for sm_100a (no name clash with the reference's NE / HC / ... globals, every
replacement call type-checks at StageGpu::record_forward, src/wzy_stage_v2.cuh:476-857, and
PrefillStageCtx::run_stage_prefill, src/wzy_prefill_tc.cuh:546-1058). Needs the reference sources:
$WZYB_REFERENCE, or a checkout named `reference` beside this repository.
GPU: the unit as built by build() (oracle/_ref/libwzydropin.so, linked against libwzyb200.so) runs
gr_read_fused's replacement on Dev buffers; its output equals the library's own entry point bit for bit
and the reference's fused_gr_norm_multi within the fp32 tolerance of the other fp32 pins.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np
import pytest

from conftest import ROOT

NVCC = "/usr/local/cuda/bin/nvcc"
DROPIN_SO = os.path.join(ROOT, "oracle", "_ref", "libwzydropin.so")


def _reference_src():
    for root in (os.environ.get("WZYB_REFERENCE"), os.path.join(os.path.dirname(ROOT), "reference")):
        if root and os.path.isfile(os.path.join(root, "src", "wzy_stage_v2.cuh")):
            return os.path.join(root, "src")
    return None


def test_dropin_unit_compiles(tmp_path):
    src = _reference_src()
    if src is None:
        pytest.skip("reference sources not present")
    if not os.path.isfile(NVCC):
        pytest.skip("nvcc not present")
    obj = tmp_path / "dropin.o"
    cmd = [NVCC, "-O0", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-Xcompiler", "-mavx2",
           "-Xcompiler", "-mfma", "-w", "-I" + src, "-I" + os.path.join(ROOT, "include"), "-c",
           os.path.join(ROOT, "oracle", "stage_dropin.cu"), "-o", str(obj)]
    p = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr[-4000:]
    nm = subprocess.run(["nm", "-C", str(obj)], capture_output=True, text=True).stdout
    for sym in ("dropin_record_forward_sites", "dropin_prefill_sites", "dropin_ple_site", "dropin_gr_read_fused"):
        assert sym in nm, sym
    # the replacements are real calls into the library, not inlined stand-ins
    undefined = subprocess.run(["nm", "-u", str(obj)], capture_output=True, text=True).stdout
    for sym in ("wzyb_gr_norm_f32", "wzyb_qk_rope_kv_append_f32", "wzyb_gdn_gated_norm_f32_f16",
                "wzyb_swiglu_interleaved_f32_f16", "wzyb_ple_gather_fp8_f32", "wzyb_embed_gather_bf16_f32"):
        assert sym in undefined, sym


@pytest.mark.gpu
def test_dropin_gr_read_fused_on_dev_buffers(orc, wz):
    import torch

    if not os.path.isfile(DROPIN_SO):
        pytest.skip("oracle/_ref/libwzydropin.so not built (needs the reference sources at build time)")
    if not orc.ref_available():
        pytest.skip("oracle/_ref/libwzyref.so not built")
    wz.lib()  # the product library first, so the drop-in unit binds to the same copy
    d = ctypes.CDLL(DROPIN_SO)
    d.dropin_gr_read_fused.restype = ctypes.c_int
    d.dropin_gr_read_fused.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                       ctypes.c_void_p]
    c3 = (ctypes.c_int * 3)()
    d.dropin_constants(c3)
    ne, hc, hcd = c3[0], c3[1], c3[2]
    assert hcd == ne * hc
    ref = orc.ref_lib()
    r = np.random.default_rng(777)
    dev = "cuda:0"
    s = torch.cuda.current_stream().cuda_stream
    for T in (1, 4):  # a decode step and a verify window
        R = r.standard_normal((T * hc, ne)).astype(np.float32)
        g = (1 + 0.02 * r.standard_normal((hc, ne))).astype(np.float32)
        dg = torch.from_numpy(g).to(dev)
        dR1, dxn1 = torch.from_numpy(R).to(dev), torch.empty((T * hc, ne), dtype=torch.float32, device=dev)
        assert d.dropin_gr_read_fused(dR1.data_ptr(), dg.data_ptr(), dxn1.data_ptr(), T, s) == 0
        dR2, dxn2 = torch.from_numpy(R).to(dev), torch.empty_like(dxn1)
        wz.gr_norm_f32(dR2, dg, None, None, dxn2, T, ne, hc)
        dR3, dxn3 = torch.from_numpy(R).to(dev), torch.empty_like(dxn1)
        assert ref.ref_fused_gr_norm_multi(dR3.data_ptr(), dg.data_ptr(), None, None, dxn3.data_ptr(), T, ne, hc,
                                           1e-6, s) == 0
        torch.cuda.synchronize()
        assert np.array_equal(dxn1.cpu().numpy(), dxn2.cpu().numpy())
        assert np.array_equal(dR1.cpu().numpy(), R)  # no pending residual: R is only read
        np.testing.assert_allclose(dxn1.cpu().numpy(), dxn3.cpu().numpy(), rtol=2e-6, atol=2e-6)
