// launch.hpp -- host-side helpers shared by the C-ABI launchers.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

#include "../../include/wzyb200.h"

namespace wzyb {

struct DeviceInfo {
    int device = -1;
    int sms = 0;
    int max_smem_optin = 0;  // bytes of dynamic shared memory one CTA may opt into
};

// Per-device facts, cached after the first query. Returns WZYB_OK or WZYB_ERR_DEVICE.
int device_info(DeviceInfo* out);

// Opt `kernel` into `bytes` of dynamic shared memory on the current device (once per device).
int ensure_smem(const void* kernel, int bytes);

// Launch tuning knobs (CTAs per SM and ring depth) per kernel family.
enum KernelFamily : int {
    kFamNorm = 0,      // residual add + RMSNorm
    kFamHeadRope = 1,  // per-head norm + RoPE
    kFamGdn = 2,       // GDN gated norm
    kFamSwiglu = 3,    // SwiGLU
    kFamGather = 4,    // embedding / PLE gathers
    kFamBundle = 5,    // layer bundles (one launch per bundle, or the ops as separate launches)
    kFamKv = 6,        // KV append (with k norm + RoPE and optional q heads)
    kFamCount = 7
};
struct Tuning {
    int ctas_per_sm;
    int stages;  // 0 = as many as the shared-memory budget allows
};
Tuning tuning(int family);
// WZYB_VARIANT_* chosen for a family (AUTO unless set by wzyb_set_kernel_variant).
int variant(int family);

// Resident CTAs per SM of `kernel` at `threads` threads and `smem` dynamic bytes on the current
// device (cached per kernel and device; at least 1).
int resident_ctas(const void* kernel, int threads, int smem);

// Persistent grid for a kernel whose CTAs loop over work: every SM filled once, never more CTAs
// than there is work for.
inline int persistent_grid(const DeviceInfo& di, int ctas_per_sm, int64_t ctas_of_work) {
    const int64_t want = (int64_t)di.sms * ctas_per_sm;
    const int64_t g = ctas_of_work < want ? ctas_of_work : want;
    return g < 1 ? 1 : (int)g;
}

// Shared-memory budget for one SM's worth of ring stages (bytes), leaving headroom for the L1.
constexpr int kSmemPerSm = 200 * 1024;

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Kernel launch with programmatic stream serialization (PDL; see pdl_begin in common.cuh), through
// cudaLaunchKernelEx. WZYB_PDL=0 in the environment launches without the attribute (plain stream
// order, for A/B measurement). A failed launch is kept for launch_status() in this thread.
bool pdl_enabled();
inline cudaError_t& launch_error_slot() {
    static thread_local cudaError_t e = cudaSuccess;
    return e;
}
template <typename... KArgs, typename... Args>
inline void launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                     Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
    if (e != cudaSuccess && launch_error_slot() == cudaSuccess) launch_error_slot() = e;
}

inline int launch_status() {
    cudaError_t e = cudaGetLastError();
    if (launch_error_slot() != cudaSuccess) {
        if (e == cudaSuccess) e = launch_error_slot();
        launch_error_slot() = cudaSuccess;
    }
    return e == cudaSuccess ? WZYB_OK : static_cast<int>(e);
}

}  // namespace wzyb
