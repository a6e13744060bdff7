// runtime.cu -- per-device set-up, the device fault word, tuning knobs and status strings.
#include <atomic>
#include <mutex>
#include <map>
#include <set>
#include <tuple>
#include <utility>

#include <cstdlib>

#include "common.cuh"
#include "launch.hpp"

namespace wzyb {

namespace {

constexpr int kMaxDevices = 64;

struct DevSlot {
    std::atomic<int> state{0};  // 0 = unknown, 1 = ok, 2 = not a supported device
    int sms = 0;
    int max_smem_optin = 0;
};
DevSlot g_dev[kMaxDevices];
std::mutex g_dev_mu;

std::mutex g_smem_mu;
std::set<std::pair<const void*, int>> g_smem_done;  // (kernel, device)

std::atomic<int> g_tune_ctas[kFamCount] = {{2}, {1}, {1}, {4}, {2}, {1}, {16}};
std::atomic<int> g_tune_stages[kFamCount] = {{0}, {0}, {0}, {0}, {0}, {0}, {0}};
std::atomic<int> g_variant[kFamCount] = {{0}, {0}, {0}, {0}, {0}, {0}, {0}};

}  // namespace

int device_info(DeviceInfo* out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return WZYB_ERR_DEVICE;
    }
    DevSlot& s = g_dev[dev];
    int st = s.state.load(std::memory_order_acquire);
    if (st == 0) {
        std::lock_guard<std::mutex> lk(g_dev_mu);
        st = s.state.load(std::memory_order_relaxed);
        if (st == 0) {
            int major = 0, sms = 0, optin = 0;
            const bool ok = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) == cudaSuccess &&
                            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess &&
                            cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) ==
                                cudaSuccess;
            cudaGetLastError();
            s.sms = sms;
            s.max_smem_optin = optin;
            st = (ok && major == 10 && sms > 0) ? 1 : 2;
            s.state.store(st, std::memory_order_release);
        }
    }
    if (st != 1) return WZYB_ERR_DEVICE;
    out->device = dev;
    out->sms = s.sms;
    out->max_smem_optin = s.max_smem_optin;
    return WZYB_OK;
}

int ensure_smem(const void* kernel, int bytes) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return WZYB_ERR_DEVICE;
    std::lock_guard<std::mutex> lk(g_smem_mu);
    const auto key = std::make_pair(kernel, dev);
    if (g_smem_done.count(key)) return WZYB_OK;
    DeviceInfo di;
    const int rc = device_info(&di);
    if (rc != WZYB_OK) return rc;
    const cudaError_t e =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, di.max_smem_optin);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return static_cast<int>(e);
    }
    (void)bytes;
    g_smem_done.insert(key);
    return WZYB_OK;
}

bool pdl_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("WZYB_PDL");
        return !(e != nullptr && e[0] == '0');
    }();
    return on;
}

Tuning tuning(int family) {
    Tuning t;
    t.ctas_per_sm = g_tune_ctas[family].load(std::memory_order_relaxed);
    t.stages = g_tune_stages[family].load(std::memory_order_relaxed);
    return t;
}

int variant(int family) { return g_variant[family].load(std::memory_order_relaxed); }

namespace {
std::mutex g_occ_mu;
std::map<std::tuple<const void*, int, int, int>, int> g_occ;  // (kernel, device, threads, smem)
}  // namespace

int resident_ctas(const void* kernel, int threads, int smem) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return 1;
    }
    std::lock_guard<std::mutex> lk(g_occ_mu);
    const auto key = std::make_tuple(kernel, dev, threads, smem);
    auto it = g_occ.find(key);
    if (it != g_occ.end()) return it->second;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, (size_t)smem) != cudaSuccess || n < 1) {
        cudaGetLastError();
        n = 1;
    }
    g_occ[key] = n;
    return n;
}

}  // namespace wzyb

extern "C" {

int wzyb_prepare_device(void) {
    wzyb::DeviceInfo di;
    return wzyb::device_info(&di);
}

int wzyb_read_faults(uint32_t* faults, int clear) {
    if (!faults) return WZYB_ERR_NULL;
    wzyb::DeviceInfo di;
    const int rc = wzyb::device_info(&di);
    if (rc != WZYB_OK) return rc;
    unsigned int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, wzyb::g_fault_word, sizeof(v));
    if (e == cudaSuccess && clear) {
        const unsigned int zero = 0;
        e = cudaMemcpyToSymbol(wzyb::g_fault_word, &zero, sizeof(zero));
    }
    if (e != cudaSuccess) return static_cast<int>(e);
    *faults = v;
    return WZYB_OK;
}

int wzyb_set_launch_tuning(int family, int ctas_per_sm, int stages) {
    if (family < 0 || family >= wzyb::kFamCount) return WZYB_ERR_VALUE;
    if (ctas_per_sm < 1 || ctas_per_sm > 16 || stages < 0 || stages > 64) return WZYB_ERR_VALUE;
    wzyb::g_tune_ctas[family].store(ctas_per_sm);
    wzyb::g_tune_stages[family].store(stages);
    return WZYB_OK;
}

int wzyb_set_kernel_variant(int family, int variant) {
    if (family < 0 || family >= wzyb::kFamCount) return WZYB_ERR_VALUE;
    if (variant < WZYB_VARIANT_AUTO || variant > WZYB_VARIANT_SPLIT) return WZYB_ERR_VALUE;
    wzyb::g_variant[family].store(variant);
    return WZYB_OK;
}

const char* wzyb_status_string(int status) {
    switch (status) {
        case WZYB_OK: return "ok";
        case WZYB_ERR_NULL: return "a required pointer is NULL";
        case WZYB_ERR_ALIGN: return "a pointer, row or head start is not 16-byte aligned";
        case WZYB_ERR_SHAPE: return "a size is out of the supported range or inconsistent";
        case WZYB_ERR_DEVICE: return "the current device is not an sm_100 (B200) GPU";
        case WZYB_ERR_VALUE: return "unknown mode / enum value";
        default: break;
    }
    if (status > 0) return cudaGetErrorString(static_cast<cudaError_t>(status));
    return "unknown status";
}

int wzyb_version(void) { return 100; }

}  // extern "C"
