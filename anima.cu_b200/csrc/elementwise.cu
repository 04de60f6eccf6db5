// elementwise.cu -- GELU / SiLU / add / mul / broadcast modulate and gate kernels (sm_100a).
//
// One kernel template covers them all: NS streamed bf16 inputs (1 or 2) read as 16-byte
// chunks with L1-bypassing loads, NB broadcast vectors (0..2) indexed by column
// (element % D, read through L1), and an Op that maps fp32 inputs to one fp32 output. Each
// thread keeps U chunks per input in flight. The grid covers the tensor once: each CTA owns
// U * 256 consecutive chunks and retires when they are stored (short-lived CTAs measured
// faster than one resident wave striding over the tensor: at 8192 x 2048 the broadcast
// residual gate went from 17.05 to 16.46 us, a plain bias add from 12.6 to 12.0 us).
// Elements past the last full chunk, and every element when a pointer is not 16-byte
// aligned, take a scalar path inside the same launch.
//
// The per-element arithmetic is the reference's own expression for each op (file:line
// at each Op), so results are bit-identical to the reference kernels.
//
// GELU and SiLU on large tensors: the output is a function of the input's 16 bits, so each
// has a 65536-entry table of bf16(F(x)) -- the reference formula at every bf16 value, filled
// on the device by the exact code path -- and the kernel becomes a table lookup from shared
// memory: one CTA of 1024 threads per SM copies the 128 KB table in (before waiting on the
// previous kernel) and streams the tensor. This replaced per-element ex2/rcp approximations
// with an exact-formula fallback: no MUFU work, no divergent fallback lanes, 4 instructions
// per element. Smaller or unaligned tensors, and calls made while a stream is being captured
// before the table exists, use the table-free kernel (fast_act_kernel), with the same results.
#include "common.cuh"
#include "tma.cuh"
#include "activation.cuh"

#include <atomic>
#include <mutex>
#include <type_traits>

namespace anima {
namespace {

constexpr int kEwBlock = 256;

struct OpGelu {  // gelu.cu:12-34
    static constexpr int NS = 1, NB = 0;
    __device__ float operator()(const float (&s)[2], const float (&)[2]) const { return gelu_tanh_f(s[0]); }
};
struct OpGeluBias {  // gelu.cu:37-64
    static constexpr int NS = 1, NB = 1;
    __device__ float operator()(const float (&s)[2], const float (&b)[2]) const {
        return gelu_tanh_f(s[0] + b[0]);
    }
};
struct OpSilu {  // silu.cu:7-24
    static constexpr int NS = 1, NB = 0;
    __device__ float operator()(const float (&s)[2], const float (&)[2]) const { return silu_f(s[0]); }
};
struct OpSiluBias {  // silu.cu:26-47
    static constexpr int NS = 1, NB = 1;
    __device__ float operator()(const float (&s)[2], const float (&b)[2]) const { return silu_f(s[0] + b[0]); }
};
struct OpAdd {  // elementwise.cu:37-53
    static constexpr int NS = 2, NB = 0;
    __device__ float operator()(const float (&s)[2], const float (&)[2]) const { return s[0] + s[1]; }
};
struct OpMul {  // elementwise.cu:125-141
    static constexpr int NS = 2, NB = 0;
    __device__ float operator()(const float (&s)[2], const float (&)[2]) const { return s[0] * s[1]; }
};
struct OpSwiGLU {  // silu.cu:7-24 on gate, rounded to bf16, then elementwise.cu:125-141
    static constexpr int NS = 2, NB = 0;
    __device__ float operator()(const float (&s)[2], const float (&)[2]) const {
        return bf16_round(silu_f(s[0])) * s[1];
    }
};
struct OpGatedGelu {  // gemma_ops.cu:5-22 (scalar formula; nvcc folds the cubic into an fma)
    static constexpr int NS = 2, NB = 0;
    __device__ float operator()(const float (&s)[2], const float (&)[2]) const {
        const float g = s[0];
        const float inner = 0.7978845608f * __fmaf_rn(0.044715f * g * g, g, g);
        return (0.5f * g * (1.0f + tanhf(inner))) * s[1];
    }
};
struct OpBiasAdd {  // elementwise.cu:184-213: x + bias[d]
    static constexpr int NS = 1, NB = 1;
    __device__ float operator()(const float (&s)[2], const float (&b)[2]) const { return s[0] + b[0]; }
};
struct OpScaleShift {  // elementwise.cu:216-236: fma(x, 1+scale[d], shift[d])
    static constexpr int NS = 1, NB = 2;
    __device__ float operator()(const float (&s)[2], const float (&b)[2]) const {
        return __fmaf_rn(s[0], 1.0f + b[0], b[1]);
    }
};
struct OpResidualGate {  // elementwise.cu:249-269: fma(y, gate[d], x)
    static constexpr int NS = 2, NB = 1;
    __device__ float operator()(const float (&s)[2], const float (&b)[2]) const {
        return __fmaf_rn(s[1], b[0], s[0]);
    }
};

struct EwArgs {
    const anima_bf16 *s0, *s1;  // streamed inputs
    const anima_bf16 *b0, *b1;  // broadcast vectors [D]
    anima_bf16 *out;
    int64_t n;       // elements to process
    int D;           // broadcast period (elements); 0 when NB == 0
    bool vec;        // 16-byte path usable
};

__device__ __forceinline__ float ldb(const anima_bf16 *p) {
    return __bfloat162float(*reinterpret_cast<const __nv_bfloat16 *>(p));
}

template <class Op, int U>
__global__ void __launch_bounds__(kEwBlock) ew_kernel(EwArgs a, Op op) {
    pdl_wait();
    constexpr int NS = Op::NS, NB = Op::NB;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    int64_t done = 0;  // elements covered by the vector loop
    if (a.vec) {
        const int64_t nch = a.n >> 3;
        done = nch << 3;
        const uint32_t dch = NB ? (uint32_t)(a.D >> 3) : 1u;
        const uint32_t cstep = NB ? (uint32_t)kEwBlock % dch : 0u;  // < dch
        // one group of U * kEwBlock consecutive chunks per CTA, chunk u of a thread at
        // threadIdx.x + u * kEwBlock (coalesced); the grid normally covers every group once
        for (int64_t base = (int64_t)blockIdx.x * kEwBlock * U + threadIdx.x; base < nch;
             base += (int64_t)gridDim.x * kEwBlock * U) {
            Vec8 in[U][NS > 1 ? 2 : 1];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int64_t i = base + u * kEwBlock;
                if (i < nch) {
                    in[u][0] = ld_stream(a.s0 + i * 8);
                    if constexpr (NS > 1) in[u][NS - 1] = ld_stream(a.s1 + i * 8);
                }
            }
            // column chunk of the thread's first chunk: one division per group (32-bit below
            // 2^32 chunks), then advanced by kEwBlock with one compare-subtract per chunk. A
            // 64-bit modulo per chunk had cost ~60 instructions of ~110 per chunk.
            uint32_t c = 0;
            if constexpr (NB > 0)
                c = base < 4294967296ll ? (uint32_t)base % dch : (uint32_t)((uint64_t)base % dch);
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int64_t i = base + u * kEwBlock;
                if (i >= nch) break;
                float f0[8], f1[8], g0[8], g1[8];
                unpack8(in[u][0], f0);
                if constexpr (NS > 1) unpack8(in[u][NS - 1], f1);
                if constexpr (NB > 0) {
                    unpack8(ld_cached(a.b0 + (int64_t)c * 8), g0);
                    if constexpr (NB > 1) unpack8(ld_cached(a.b1 + (int64_t)c * 8), g1);
                    c += cstep;
                    if (c >= dch) c -= dch;
                }
                float r[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    float s[2] = {f0[e], NS > 1 ? f1[e] : 0.0f};
                    float b[2] = {NB > 0 ? g0[e] : 0.0f, NB > 1 ? g1[e] : 0.0f};
                    r[e] = op(s, b);
                }
                st_vec(a.out + i * 8, pack8(r));
            }
        }
    }
    pdl_launch();
    // Scalar path: the tail past the last full chunk, or everything when misaligned.
    for (int64_t e = done + tid; e < a.n; e += stride) {
        float s[2] = {ldb(a.s0 + e), NS > 1 ? ldb(a.s1 + e) : 0.0f};
        float b[2] = {0.0f, 0.0f};
        if constexpr (NB > 0) {
            const int64_t d = e % a.D;
            b[0] = ldb(a.b0 + d);
            if constexpr (NB > 1) b[1] = ldb(a.b1 + d);
        }
        *reinterpret_cast<__nv_bfloat16 *>(a.out + e) = __float2bfloat16_rn(op(s, b));
    }
}

template <class Op>
int launch_ew(const EwArgs &a, cudaStream_t stream) {
    if (a.n <= 0) return ANIMA_OK;
    constexpr int U = Op::NS > 1 ? 2 : 4;
    const int64_t work = a.vec ? ((a.n >> 3) + U - 1) / U : a.n;  // threads
    int64_t blocks = (work + kEwBlock - 1) / kEwBlock;
    if (blocks < 1) blocks = 1;                    // fewer than 8 elements: the scalar tail
    if (blocks > 2147483647) blocks = 2147483647;  // the kernel strides over the rest
    launch(ew_kernel<Op, U>, (unsigned)blocks, kEwBlock, 0, stream, a, Op{});
    return launch_status();
}

template <class F>
__device__ __noinline__ uint32_t exact_bf16(uint32_t b) {  // out of line, for the ragged tail
    return exact_bits<F>(b);
}

// U chunks per thread and group, groups grid-strided; the next group's loads are issued
// before the current group is computed, so every thread keeps U 16-byte loads in flight.
template <int U, int NS>
__device__ __forceinline__ void load_group(Vec8 (&in)[U][NS], const EwArgs &a, int64_t base, int64_t stride,
                                           int64_t nch) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const int64_t i = base + u * stride;
        if (i < nch) {
            in[u][0] = ld_stream(a.s0 + i * 8);
            if constexpr (NS > 1) in[u][1] = ld_stream(a.s1 + i * 8);
        }
    }
}

template <class F, int U, int NS>
__device__ __forceinline__ void act_group(const Vec8 (&in)[U][NS], const EwArgs &a, int64_t base, int64_t stride,
                                          int64_t nch) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const int64_t i = base + u * stride;
        if (i >= nch) break;
        Vec8 o = fast_chunk<F>(in[u][0]);
        if constexpr (NS > 1) {  // elementwise.cu:138-140: product of the bf16 silu value and up
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t uw = in[u][1].w[j];
                const float2 p = __fmul2_rn(make_float2(bf_lo(o.w[j]), bf_hi(o.w[j])), make_float2(bf_lo(uw), bf_hi(uw)));
                o.w[j] = pack_bf2(p.x, p.y);
            }
        }
        st_vec(a.out + i * 8, o);
    }
}

// NS = 1: out = F(x). NS = 2 (SwiGLU): out = bf16(F(gate)) * up, as silu_bf16 then mul_bf16.
template <class F, int NS>
__global__ void __launch_bounds__(kEwBlock, NS == 1 ? 6 : 2) fast_act_kernel(EwArgs a) {
    pdl_wait();
    constexpr int U = 2;  // chunks per group (x2 in flight); swept 2-4 x 4-8 CTAs per SM
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t nch = a.vec ? a.n >> 3 : 0;
    Vec8 x0[U][NS], x1[U][NS];
    const int64_t step = stride * U;
    load_group<U, NS>(x0, a, tid, stride, nch);
    for (int64_t base = tid; base < nch;) {  // unrolled by two so the buffers alternate without copies
        load_group<U, NS>(x1, a, base + step, stride, nch);
        act_group<F, U, NS>(x0, a, base, stride, nch);
        base += step;
        if (base >= nch) break;
        load_group<U, NS>(x0, a, base + step, stride, nch);
        act_group<F, U, NS>(x1, a, base, stride, nch);
        base += step;
    }
    pdl_launch();
    for (int64_t e = (nch << 3) + tid; e < a.n; e += stride) {
        const uint32_t r = exact_bf16<F>(*reinterpret_cast<const uint16_t *>(a.s0 + e));
        if constexpr (NS == 1) {
            a.out[e] = (anima_bf16)r;
        } else {
            const float up = __bfloat162float(*reinterpret_cast<const __nv_bfloat16 *>(a.s1 + e));
            *reinterpret_cast<__nv_bfloat16 *>(a.out + e) = __float2bfloat16_rn(__uint_as_float(r << 16) * up);
        }
    }
}

template <class F, int NS>
int launch_fast_act(const EwArgs &a, cudaStream_t stream) {
    if (a.n <= 0) return ANIMA_OK;
    const int64_t work = a.vec ? ((a.n >> 3) + 1) / 2 : a.n;
    int err = ANIMA_OK;
    const unsigned blocks = wave_grid((const void *)fast_act_kernel<F, NS>, kEwBlock, 0, work, &err);
    if (err) return err;
    launch(fast_act_kernel<F, NS>, blocks, kEwBlock, 0, stream, a);
    return launch_status();
}

// ------------------------------------------------------------ activation tables
// bf16(F(x)) for every bf16 bit pattern x: [0] GELU-tanh, [1] SiLU. Static device memory of
// the module (one copy per device); filled by fill_act_table on the first table-path call.
__device__ __align__(256) uint16_t g_act_table[2][65536];
constexpr int kTabEntries = 65536;
constexpr int kTabBytes = kTabEntries * 2;
constexpr int kTabBlock = 1024;   // one CTA per SM: the table takes 128 KB of shared memory
constexpr int64_t kTabMinElems = 1 << 20;

template <class F>
__global__ void fill_act_table(uint16_t *table) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < kTabEntries) table[i] = (uint16_t)exact_bits<F>(i);
}

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}

template <int U>
__device__ __forceinline__ void lookup_group(const Vec8 (&in)[U][1], const EwArgs &a, const uint16_t *tab,
                                             int64_t base, int64_t stride, int64_t nch) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const int64_t i = base + u * stride;
        if (i >= nch) break;
        Vec8 o;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t w = in[u][0].w[j];
            o.w[j] = (uint32_t)tab[w & 0xffffu] | ((uint32_t)tab[w >> 16] << 16);
        }
        st_vec(a.out + i * 8, o);
    }
}

// The table kernel below 2^26 elements: every thread keeps two 16-byte loads in flight in
// registers (double buffered), grid-strided over the tensor.
__global__ void __launch_bounds__(kTabBlock, 1) table_act_regs(EwArgs a, const uint16_t *__restrict__ table) {
    extern __shared__ __align__(16) uint16_t tab[];
    // The table does not depend on the previous kernel: copy it in before waiting on it.
    for (int q = threadIdx.x; q < kTabEntries / 8; q += kTabBlock) cp_async16(tab + q * 8, table + q * 8);
    asm volatile("cp.async.commit_group;" ::: "memory");
    pdl_wait();
    constexpr int U = 2;  // swept 1-4: 2 is best (43.5 us on [8192, 8192])
    const int64_t tid = (int64_t)blockIdx.x * kTabBlock + threadIdx.x, stride = (int64_t)gridDim.x * kTabBlock;
    const int64_t nch = a.n >> 3, step = stride * U;
    Vec8 x0[U][1], x1[U][1];
    load_group<U, 1>(x0, a, tid, stride, nch);
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    for (int64_t base = tid; base < nch;) {
        load_group<U, 1>(x1, a, base + step, stride, nch);
        lookup_group<U>(x0, a, tab, base, stride, nch);
        base += step;
        if (base >= nch) break;
        load_group<U, 1>(x0, a, base + step, stride, nch);
        lookup_group<U>(x1, a, tab, base, stride, nch);
        base += step;
    }
    pdl_launch();
    for (int64_t e = (nch << 3) + tid; e < a.n; e += stride)
        reinterpret_cast<uint16_t *>(a.out)[e] = tab[reinterpret_cast<const uint16_t *>(a.s0)[e]];
}

// The table kernel's input stream: 1-D bulk copies (the TMA unit; this GPU's memory only, no
// multicast) of kTabStageBytes blocks into kTabStages shared-memory stages beside the table,
// each completing on its own mbarrier. Blocks go round-robin over the CTAs (one per SM); thread
// t turns chunk t of a block into chunk t of the output. Thread 0 refills the stage of the
// previous block once all 1024 threads have released it (an "empty" mbarrier), so up to six
// 16 KB blocks (96 KB, all the shared memory the table leaves) are in flight per SM without
// holding registers: 42.1 against 43.7 us on the DiT FFN's [8192, 8192] for the previous
// form, which kept two 16-byte loads per thread in flight in registers (five stages: 44.1 us,
// four: 48.3 us). Below 2^26 elements table_act_regs stays faster (22.8 against 23.4 us at
// [4096, 8192]: with ~28 blocks per SM the CTA-wide hand-off of each stage weighs more).
// Every wait is bounded; one that runs out is counted (ew_wait_timeouts).
constexpr int64_t kTabTmaMinElems = (int64_t)1 << 26;
constexpr int kTabStages = 6;
constexpr int kTabStageBytes = 16384;                 // one 16-byte chunk per thread
constexpr int kTabStageChunks = kTabStageBytes / 16;
constexpr int kTabSmem = kTabBytes + kTabStages * kTabStageBytes + kTabStages * 16;
static_assert(kTabStageChunks == kTabBlock, "one chunk per thread and stage");

__device__ unsigned int g_ew_wait_timeouts;

__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__global__ void __launch_bounds__(kTabBlock, 1) table_act_kernel(EwArgs a, const uint16_t *__restrict__ table) {
    extern __shared__ __align__(1024) unsigned char tab_smem[];
    uint16_t *tab = reinterpret_cast<uint16_t *>(tab_smem);
    unsigned char *stages = tab_smem + kTabBytes;
    uint64_t *full = reinterpret_cast<uint64_t *>(stages + kTabStages * kTabStageBytes);
    uint64_t *empty = full + kTabStages;
    const int tid = threadIdx.x;
    // The table does not depend on the previous kernel: copy it in before waiting on it.
    for (int q = tid; q < kTabEntries / 8; q += kTabBlock) cp_async16(tab + q * 8, table + q * 8);
    asm volatile("cp.async.commit_group;" ::: "memory");
    if (tid == 0) {
        for (int st = 0; st < kTabStages; ++st) {
            mbar_init(&full[st], 1);
            mbar_init(&empty[st], kTabBlock);
        }
        mbar_fence_init();
    }
    __syncthreads();
    pdl_wait();
    const int64_t nch = a.n >> 3;
    const int64_t nblk = (nch + kTabStageChunks - 1) / kTabStageChunks;
    const int my = blockIdx.x < nblk ? (int)((nblk - 1 - blockIdx.x) / gridDim.x + 1) : 0;
    auto issue = [&](int k) {  // thread 0: the CTA's k-th block into stage k % kTabStages
        const int64_t blk = blockIdx.x + (int64_t)k * gridDim.x;
        const int64_t left = nch - blk * kTabStageChunks;
        const uint32_t bytes = (uint32_t)((left < kTabStageChunks ? left : kTabStageChunks) * 16);
        const int st = k % kTabStages;
        mbar_arrive_expect_tx(&full[st], bytes);
        bulk_load(stages + (size_t)st * kTabStageBytes, a.s0 + blk * kTabStageChunks * 8, bytes, &full[st]);
    };
    if (tid == 0)
        for (int k = 0; k < kTabStages && k < my; ++k) issue(k);
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();  // the table is in shared memory
    bool ok = true;
    for (int k = 0; k < my; ++k) {
        const int st = k % kTabStages;
        if (!mbar_wait(&full[st], (uint32_t)(k / kTabStages) & 1u)) {
            ok = false;
            break;
        }
        const int64_t blk = blockIdx.x + (int64_t)k * gridDim.x;
        if (blk * kTabStageChunks + tid < nch) {
            const Vec8 in = reinterpret_cast<const Vec8 *>(stages + (size_t)st * kTabStageBytes)[tid];
            Vec8 o;
#pragma unroll
            for (int j = 0; j < 4; ++j) o.w[j] = (uint32_t)tab[in.w[j] & 0xffffu] | ((uint32_t)tab[in.w[j] >> 16] << 16);
            st_vec(a.out + (blk * kTabStageChunks + tid) * 8, o);
        }
        mbar_arrive(&empty[st]);
        if (tid == 0 && k >= 1 && k - 1 + kTabStages < my) {
            // the previous block's stage, once every thread has read it
            if (mbar_wait(&empty[(k - 1) % kTabStages], (uint32_t)((k - 1) / kTabStages) & 1u)) issue(k - 1 + kTabStages);
            else ok = false;
        }
    }
    if (!ok) atomicAdd(&g_ew_wait_timeouts, 1u);
    pdl_launch();
    const int64_t stride = (int64_t)gridDim.x * kTabBlock;
    for (int64_t e = (nch << 3) + (int64_t)blockIdx.x * kTabBlock + tid; e < a.n; e += stride)
        reinterpret_cast<uint16_t *>(a.out)[e] = tab[reinterpret_cast<const uint16_t *>(a.s0)[e]];
}

constexpr int kTabDevices = 64;
std::atomic<uintptr_t> g_table_addr[kTabDevices];  // device address of g_act_table (set before a ready bit)
std::atomic<unsigned> g_table_ready[kTabDevices];  // bit t set = table t filled on that device
std::mutex g_table_fill_mu[kTabDevices];           // one first fill per device and table at a time

// The device's table `t`, filled if it is not yet and the stream is not being captured
// (filling launches on `stream` and waits for it, once per device). Null: use the
// table-free kernel. *err receives a CUDA error from the fill. While a capture is under way
// nothing but the capture query runs here, so a capture is never disturbed.
template <class F>
const uint16_t *act_table(int t, cudaStream_t stream, int *err) {
    *err = ANIMA_OK;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev >= kTabDevices) {
        cudaGetLastError();
        return nullptr;
    }
    if (g_table_ready[dev].load(std::memory_order_acquire) & (1u << t))
        return reinterpret_cast<const uint16_t *>(g_table_addr[dev].load(std::memory_order_acquire)) + t * kTabEntries;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
        cudaGetLastError();
        return nullptr;
    }
    // Threads making a first call on this device at the same time: one fills, the others
    // wait here and then find the ready bit set (no second fill, no fill over a table that
    // another thread's kernel is already reading).
    std::lock_guard<std::mutex> lock(g_table_fill_mu[dev]);
    if (g_table_ready[dev].load(std::memory_order_acquire) & (1u << t))
        return reinterpret_cast<const uint16_t *>(g_table_addr[dev].load(std::memory_order_acquire)) + t * kTabEntries;
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_act_table) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    g_table_addr[dev].store((uintptr_t)p, std::memory_order_release);
    uint16_t *table = static_cast<uint16_t *>(p) + t * kTabEntries;
    fill_act_table<F><<<kTabEntries / 256, 256, 0, stream>>>(table);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) {
        *err = (int)e;
        return nullptr;
    }
    g_table_ready[dev].fetch_or(1u << t, std::memory_order_acq_rel);
    return table;
}

template <class F>
int launch_act(const EwArgs &a, cudaStream_t stream, int t) {
    if (a.vec && a.n >= kTabMinElems) {
        int err = ANIMA_OK;
        const uint16_t *table = act_table<F>(t, stream, &err);
        if (err) return err;
        if (table) {
            if (a.n >= kTabTmaMinElems) {
                if (int e = allow_dynamic_smem((const void *)table_act_kernel, kTabSmem, 8)) return e;
                launch(table_act_kernel, (unsigned)sm_count(), kTabBlock, kTabSmem, stream, a, table);
            } else {
                if (int e = allow_dynamic_smem((const void *)table_act_regs, kTabBytes, 9)) return e;
                launch(table_act_regs, (unsigned)sm_count(), kTabBlock, kTabBytes, stream, a, table);
            }
            return launch_status();
        }
    }
    return launch_fast_act<F, 1>(a, stream);
}

bool bf16_ok(const void *p) { return aligned_to(p, 2); }

// Validates and launches a flat op over n elements (n = 2*floor(N/2), as the reference's
// pair loop covers).
template <class Op>
int flat_op(const anima_bf16 *s0, const anima_bf16 *s1, const anima_bf16 *bias, anima_bf16 *out,
            int64_t N, int D, cudaStream_t stream) {
    constexpr int NS = Op::NS, NB = Op::NB;
    if (N < 0) return ANIMA_ERR_BAD_SHAPE;
    if (NB > 0 && (D <= 0 || (D & 1))) return ANIMA_ERR_BAD_SHAPE;
    const int64_t n = N / 2 * 2;
    if (n == 0) return ANIMA_OK;
    if (!s0 || !out || (NS > 1 && !s1) || (NB > 0 && !bias)) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(s0) || !bf16_ok(out) || (NS > 1 && !bf16_ok(s1)) || (NB > 0 && !bf16_ok(bias)))
        return ANIMA_ERR_MISALIGNED;
    if (n > INT64_MAX / 2) return ANIMA_ERR_TOO_LARGE;
    if (partial_overlap(s0, n * 2, out, n * 2) || (NS > 1 && partial_overlap(s1, n * 2, out, n * 2)))
        return ANIMA_ERR_OVERLAP;
    EwArgs a{s0, NS > 1 ? s1 : nullptr, NB > 0 ? bias : nullptr, nullptr, out, n, NB > 0 ? D : 0, false};
    a.vec = aligned16(s0) && aligned16(out) && (NS < 2 || aligned16(s1)) &&
            (NB == 0 || (aligned16(bias) && D % 8 == 0));
    if constexpr (std::is_same<Op, OpGelu>::value) return launch_act<GeluF>(a, stream, 0);
    if constexpr (std::is_same<Op, OpSilu>::value) return launch_act<SiluF>(a, stream, 1);
    if constexpr (std::is_same<Op, OpSwiGLU>::value) return launch_fast_act<SiluF, 2>(a, stream);
    return launch_ew<Op>(a, stream);
}

// Validates and launches a row-broadcast op over [M, D].
template <class Op>
int bcast_op(const anima_bf16 *x, const anima_bf16 *y, const anima_bf16 *b0, const anima_bf16 *b1,
             anima_bf16 *out, int M, int D, cudaStream_t stream) {
    constexpr int NS = Op::NS, NB = Op::NB;
    if (M < 0 || D <= 0 || (D & 1)) return ANIMA_ERR_BAD_SHAPE;
    const int64_t n = (int64_t)M * D;
    if (n == 0) return ANIMA_OK;
    if (!x || !out || (NS > 1 && !y) || !b0 || (NB > 1 && !b1)) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(x) || !bf16_ok(out) || (NS > 1 && !bf16_ok(y)) || !bf16_ok(b0) ||
        (NB > 1 && !bf16_ok(b1)))
        return ANIMA_ERR_MISALIGNED;
    if (partial_overlap(x, n * 2, out, n * 2) || (NS > 1 && partial_overlap(y, n * 2, out, n * 2)))
        return ANIMA_ERR_OVERLAP;
    EwArgs a{x, NS > 1 ? y : nullptr, b0, NB > 1 ? b1 : nullptr, out, n, D, false};
    a.vec = D % 8 == 0 && aligned16(x) && aligned16(out) && (NS < 2 || aligned16(y)) &&
            aligned16(b0) && (NB < 2 || aligned16(b1));
    return launch_ew<Op>(a, stream);
}

}  // namespace
}  // namespace anima

using namespace anima;

// ================================================================ C ABI

extern "C" int anima_gelu_tanh_bf16(const anima_bf16 *x, anima_bf16 *out, int64_t N,
                                    anima_stream_t stream) {
    return flat_op<OpGelu>(x, nullptr, nullptr, out, N, 0, stream);
}

extern "C" int anima_gelu_tanh_bias_bf16(const anima_bf16 *x, const anima_bf16 *bias,
                                         anima_bf16 *out, int64_t N, int D, anima_stream_t stream) {
    return flat_op<OpGeluBias>(x, nullptr, bias, out, N, D, stream);
}

extern "C" int anima_silu_bf16(const anima_bf16 *x, anima_bf16 *out, int64_t N,
                               anima_stream_t stream) {
    return flat_op<OpSilu>(x, nullptr, nullptr, out, N, 0, stream);
}

extern "C" int anima_silu_bias_bf16(const anima_bf16 *x, const anima_bf16 *bias, anima_bf16 *out,
                                    int64_t N, int D, anima_stream_t stream) {
    return flat_op<OpSiluBias>(x, nullptr, bias, out, N, D, stream);
}

extern "C" int anima_add_bf16(const anima_bf16 *a, const anima_bf16 *b, anima_bf16 *out, int64_t N,
                              anima_stream_t stream) {
    return flat_op<OpAdd>(a, b, nullptr, out, N, 0, stream);
}

extern "C" int anima_mul_bf16(const anima_bf16 *a, const anima_bf16 *b, anima_bf16 *out, int64_t N,
                              anima_stream_t stream) {
    return flat_op<OpMul>(a, b, nullptr, out, N, 0, stream);
}

extern "C" int anima_swiglu_bf16(const anima_bf16 *gate, const anima_bf16 *up, anima_bf16 *out,
                                 int64_t N, anima_stream_t stream) {
    return flat_op<OpSwiGLU>(gate, up, nullptr, out, N, 0, stream);
}

extern "C" int anima_gated_gelu_bf16(const anima_bf16 *gate, const anima_bf16 *up, anima_bf16 *out,
                                     int64_t N, anima_stream_t stream) {
    // gemma_ops.cu:24-31 covers every element (no pair loop): process N, not 2*floor(N/2).
    if (N < 0) return ANIMA_ERR_BAD_SHAPE;
    if (N == 0) return ANIMA_OK;
    if (!gate || !up || !out) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(gate) || !bf16_ok(up) || !bf16_ok(out)) return ANIMA_ERR_MISALIGNED;
    if (partial_overlap(gate, N * 2, out, N * 2) || partial_overlap(up, N * 2, out, N * 2))
        return ANIMA_ERR_OVERLAP;
    EwArgs a{gate, up, nullptr, nullptr, out, N, 0, false};
    a.vec = aligned16(gate) && aligned16(up) && aligned16(out);
    return launch_ew<OpGatedGelu>(a, stream);
}

extern "C" int anima_bias_add_bf16(const anima_bf16 *x, const anima_bf16 *bias, anima_bf16 *out, int M, int D,
                                   anima_stream_t stream) {
    return bcast_op<OpBiasAdd>(x, nullptr, bias, nullptr, out, M, D, stream);
}

extern "C" int anima_scale_shift_bcast_bf16(const anima_bf16 *x, const anima_bf16 *scale,
                                            const anima_bf16 *shift, anima_bf16 *out, int M, int D,
                                            anima_stream_t stream) {
    return bcast_op<OpScaleShift>(x, nullptr, scale, shift, out, M, D, stream);
}

extern "C" int anima_residual_gate_bcast_bf16(const anima_bf16 *x, const anima_bf16 *y,
                                              const anima_bf16 *gate, anima_bf16 *out, int M, int D,
                                              anima_stream_t stream) {
    return bcast_op<OpResidualGate>(x, y, gate, nullptr, out, M, D, stream);
}

// Bounded waits of the table kernel that ran out (anima_wait_timeouts adds them in).
namespace anima {
int ew_wait_timeouts(unsigned int *count, int reset) {
    cudaError_t e = cudaMemcpyFromSymbol(count, g_ew_wait_timeouts, sizeof(unsigned int));
    if (e == cudaSuccess && reset) {
        const unsigned int zero = 0;
        e = cudaMemcpyToSymbol(g_ew_wait_timeouts, &zero, sizeof(unsigned int));
    }
    return e == cudaSuccess ? ANIMA_OK : (int)e;
}
}  // namespace anima
