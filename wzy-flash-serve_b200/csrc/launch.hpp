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
    kFamCount = 5
};
struct Tuning {
    int ctas_per_sm;
    int stages;  // 0 = as many as the shared-memory budget allows
};
Tuning tuning(int family);

// Shared-memory budget for one SM's worth of ring stages (bytes), leaving headroom for the L1.
constexpr int kSmemPerSm = 200 * 1024;

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int launch_status() {
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? WZYB_OK : static_cast<int>(e);
}

}  // namespace wzyb
