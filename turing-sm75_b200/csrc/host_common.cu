// host_common.cu -- host helpers shared by the kernels and the C ABI:
// device check, TMA descriptor encoding, status strings, device error words.
#include <atomic>
#include <cstring>

#include "common.cuh"
#include "errwords.h"

namespace b200 {

int check_device_sm100() {
    int dev = 0;
    B200_TRY_CUDA(cudaGetDevice(&dev));
    int major = 0, minor = 0;
    B200_TRY_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    B200_TRY_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev));
    if (major != 10 || minor != 0) return B200LAB_ERR_DEVICE;
    return B200LAB_OK;
}

int device_sm_count() {
    int dev = 0, v = 0;
    if (cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0)
        return v;
    return 148;
}

int causal_tail_groups(int units_per_group, int groups) {
    if (units_per_group <= 0 || groups <= 0) return 0;
    const long long want = (8LL * device_sm_count() + units_per_group - 1) / units_per_group;
    return (int)(want < groups ? want : groups);
}

// cuTensorMapEncodeTiled reached through the runtime's driver entry point, so
// the library does not link libcuda directly.
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

static std::atomic<unsigned long long> g_launches{0};

__device__ int g_err_watchdog = 0;

// One thread waits on a barrier that nothing arrives on: the bounded wait gives up after
// kWaitLimitNs and records B200LAB_ERR_TIMEOUT, as any kernel here does when a partner
// never arrives.
__global__ void watchdog_selftest_kernel() {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) mbar_wait(&bar, 0, &abort_flag, &g_err_watchdog);
}
void count_launch(int n) { g_launches.fetch_add((unsigned long long)n, std::memory_order_relaxed); }

int make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes,
                 uint64_t d0, uint64_t d1, uint64_t d2, uint32_t box0, uint32_t box1,
                 CUtensorMapSwizzle swizzle) {
    auto fn = encode_fn();
    if (!fn) return B200LAB_ERR_CUDA;
    cuuint64_t dims[3] = {d0, d1, d2};
    cuuint64_t strides[2] = {d0 * (uint64_t)elem_bytes, d0 * d1 * (uint64_t)elem_bytes};
    cuuint32_t box[3] = {box0, box1, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    std::memset(map, 0, sizeof(*map));
    CUresult r = fn(map, dtype, 3, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? B200LAB_OK : B200LAB_ERR_INVALID;
}

int make_tmap_4d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes,
                 uint64_t d0, uint64_t d1, uint64_t d2, uint64_t d3, uint32_t box0, uint32_t box1,
                 uint32_t box2, CUtensorMapSwizzle swizzle) {
    auto fn = encode_fn();
    if (!fn) return B200LAB_ERR_CUDA;
    const uint64_t e = (uint64_t)elem_bytes;
    cuuint64_t dims[4] = {d0, d1, d2, d3};
    cuuint64_t strides[3] = {d0 * e, d0 * d1 * e, d0 * d1 * d2 * e};
    cuuint32_t box[4] = {box0, box1, box2, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    std::memset(map, 0, sizeof(*map));
    CUresult r = fn(map, dtype, 4, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? B200LAB_OK : B200LAB_ERR_INVALID;
}

}  // namespace b200

B200_DEFINE_ERR_TAKER(watchdog, b200::g_err_watchdog)

extern "C" int b200lab_watchdog_selftest(void* stream) {
    int rc = b200::check_device_sm100();
    if (rc != B200LAB_OK) return rc;
    b200::watchdog_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>();
    b200::count_launch(1);
    return cudaGetLastError() == cudaSuccess ? B200LAB_OK : B200LAB_ERR_CUDA;
}

extern "C" const char* b200lab_strerror(int status) {
    switch (status) {
        case B200LAB_OK: return "ok";
        case B200LAB_ERR_INVALID: return "invalid argument (null pointer or inconsistent shape)";
        case B200LAB_ERR_UNSUPPORTED: return "unsupported configuration (not built)";
        case B200LAB_ERR_CUDA: return "CUDA runtime error";
        case B200LAB_ERR_TIMEOUT: return "device-side bounded wait timed out";
        case B200LAB_ERR_WORKSPACE: return "workspace missing or too small";
        case B200LAB_ERR_DEVICE: return "current device is not sm_100 (B200)";
        default: return "unknown status";
    }
}

extern "C" int b200lab_version(void) { return 100; /* 0.1.0 */ }

extern "C" unsigned long long b200lab_launch_count(void) {
    return b200::g_launches.load(std::memory_order_relaxed);
}

extern "C" int b200lab_device_status(void* stream) {
    if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess)
        return B200LAB_ERR_CUDA;
    int worst = B200LAB_OK;
    const int words[] = {b200::take_err_attn(), b200::take_err_attn_gated(), b200::take_err_gdn_prefill(),
                         b200::take_err_gdn_decode(), b200::take_err_watchdog()};
    for (int w : words) {
        if (w == B200LAB_ERR_CUDA) return B200LAB_ERR_CUDA;
        if (w != B200LAB_OK) worst = w;
    }
    return worst;
}
