// abi.cu -- library-wide host helpers of the C ABI: device properties, status strings.
#include <atomic>
#include <mutex>
#include <vector>

#include <cudaTypedefs.h>

#include "common.cuh"
#include "tma.cuh"

namespace anima {

namespace {
constexpr int kMaxDevices = 64;
std::atomic<int> g_sm_count[kMaxDevices];          // 0 = not queried yet
std::atomic<uint64_t> g_smem_slots[kMaxDevices];   // bit i set = slot i configured
}  // namespace

int sm_count() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 148;
    if (dev >= kMaxDevices) {
        int n = 0;
        return cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0 ? n : 148;
    }
    int n = g_sm_count[dev].load(std::memory_order_relaxed);
    if (n > 0) return n;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
        cudaGetLastError();  // do not leave the query's error for launch_status() to report
        return 148;
    }
    g_sm_count[dev].store(n, std::memory_order_relaxed);
    return n;
}

int allow_dynamic_smem(const void *kernel, int bytes, int slot) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return ANIMA_ERR_NO_DEVICE;
    const uint64_t bit = 1ull << slot;
    if (dev < kMaxDevices && (g_smem_slots[dev].load(std::memory_order_acquire) & bit)) return ANIMA_OK;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return (int)e;
    if (dev < kMaxDevices) g_smem_slots[dev].fetch_or(bit, std::memory_order_acq_rel);
    return ANIMA_OK;
}

namespace {
struct OccEntry {
    int dev;
    const void *kernel;
    int block, smem, ctas;
};
std::mutex g_occ_mu;
std::vector<OccEntry> g_occ;
}  // namespace

int resident_ctas(const void *kernel, int block, int smem, int *err) {
    *err = ANIMA_OK;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        *err = ANIMA_ERR_NO_DEVICE;
        return 0;
    }
    {
        std::lock_guard<std::mutex> lock(g_occ_mu);
        for (const OccEntry &e : g_occ)
            if (e.dev == dev && e.kernel == kernel && e.block == block && e.smem == smem) return e.ctas;
    }
    cudaError_t e = cudaSuccess;
    if (smem > 48 * 1024) e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    int n = 0;
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, block, (size_t)smem);
    if (e != cudaSuccess || n <= 0) {
        cudaGetLastError();
        *err = e != cudaSuccess ? (int)e : (int)cudaErrorInvalidConfiguration;
        return 0;
    }
    std::lock_guard<std::mutex> lock(g_occ_mu);
    g_occ.push_back(OccEntry{dev, kernel, block, smem, n});
    return n;
}

namespace {
// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link), looked up
// once per process.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = []() -> PFN_cuTensorMapEncodeTiled_v12000 {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }();
    return fn;
}
}  // namespace

bool encode_bf16_map_3d(CUtensorMap *map, const void *base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1,
                        uint64_t s2, uint32_t b0, uint32_t b1) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (!encode) return false;
    const cuuint64_t dims[3] = {d0, d1, d2};
    const cuuint64_t strides[2] = {s1, s2};
    const cuuint32_t box[3] = {b0, b1, 1};
    const cuuint32_t elem[3] = {1, 1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

unsigned wave_grid(const void *kernel, int block, int smem, int64_t work, int *err) {
    const int per_sm = resident_ctas(kernel, block, smem, err);
    if (*err) return 0;
    int64_t blocks = (work + block - 1) / block;
    const int64_t wave = (int64_t)per_sm * sm_count();
    if (blocks > wave) blocks = wave;
    return (unsigned)(blocks < 1 ? 1 : blocks);
}

}  // namespace anima

extern "C" const char *anima_status_string(int status) {
    switch (status) {
    case ANIMA_OK: return "ANIMA_OK";
    case ANIMA_ERR_NULL_POINTER: return "ANIMA_ERR_NULL_POINTER: a required pointer is NULL";
    case ANIMA_ERR_BAD_SHAPE: return "ANIMA_ERR_BAD_SHAPE: invalid size argument";
    case ANIMA_ERR_MISALIGNED: return "ANIMA_ERR_MISALIGNED: pointer not aligned to its element size";
    case ANIMA_ERR_TOO_LARGE: return "ANIMA_ERR_TOO_LARGE: size overflows the index arithmetic";
    case ANIMA_ERR_OVERLAP: return "ANIMA_ERR_OVERLAP: output partially overlaps an input";
    case ANIMA_ERR_NO_DEVICE: return "ANIMA_ERR_NO_DEVICE: no current CUDA device";
    default:
        if (status > 0) return cudaGetErrorString((cudaError_t)status);
        return "unknown anima status";
    }
}

extern "C" const char *anima_version(void) { return "anima_b200 0.1.0 sm_100a"; }
