// common.cuh -- device helpers shared by the anima_b200 kernels (sm_100a).
//
// Memory: every hot kernel moves 16-byte vectors (8 bf16) with explicit PTX loads and
// stores. Streamed tensors bypass L1 (L1::no_allocate); the small broadcast vectors
// (scale/shift/gate/weights, RoPE tables) use the default cached path.
//
// Numerics: outputs must match the reference kernels' rounding. Pair sums and sums of
// squares therefore go through `ref_pair_tree_sum`, which replays, in registers, the
// exact addition tree of the reference's one-CTA-per-row reduction.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/anima_b200.h"

namespace anima {

// ----------------------------------------------------------------- 16-byte I/O

struct alignas(16) Vec8 {
    uint32_t w[4];  // four packed bf16 pairs, element 2i in the low half of w[i]
};

// Streamed read: no L1 allocation (each byte is read once per kernel).
__device__ __forceinline__ Vec8 ld_stream(const void *p) {
    Vec8 r;
    asm volatile("ld.global.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.w[0]), "=r"(r.w[1]), "=r"(r.w[2]), "=r"(r.w[3])
                 : "l"(p));
    return r;
}

// Cached read for broadcast vectors and tables that many warps re-read.
__device__ __forceinline__ Vec8 ld_cached(const void *p) {
    Vec8 r;
    asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.w[0]), "=r"(r.w[1]), "=r"(r.w[2]), "=r"(r.w[3])
                 : "l"(p));
    return r;
}

__device__ __forceinline__ void st_vec(void *p, const Vec8 &v) {
    asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.w[0]), "r"(v.w[1]),
                 "r"(v.w[2]), "r"(v.w[3])
                 : "memory");
}

__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// x / D for a compile-time power of two D: the exact quotient equals x * 2^-k, so the
// correctly rounded product is the correctly rounded quotient (IEEE round-to-nearest, also
// for subnormal results), one multiply instead of the division sequence.
template <int D>
__device__ __forceinline__ float div_pow2(float x) {
    static_assert(D > 0 && (D & (D - 1)) == 0, "D must be a power of two");
    return __fmul_rn(x, 1.0f / (float)D);
}

// Pair sums of squares fmaf(b, b, a * a) (the reference's a*a + b*b as nvcc contracts it)
// for the bf16 pairs in words w0 and w1, on packed fp32x2 ops: each lane rounds as the
// scalar op does, at half the issue cost.
__device__ __forceinline__ float2 sq_pair2(uint32_t w0, uint32_t w1) {
    const float2 a = make_float2(bf_lo(w0), bf_lo(w1)), b = make_float2(bf_hi(w0), bf_hi(w1));
    return __ffma2_rn(b, b, __fmul2_rn(a, a));
}

// sm_100 mixed-precision fp32 arithmetic with bf16 operands taken straight from a packed pair:
// each converts its bf16 operand to fp32 exactly and rounds the fp32 result once, so the bits
// are those of the unpacked scalar op, without the unpacking instructions.
__device__ __forceinline__ float2 bf2_sub(uint32_t w, float c) {  // (lo - c, hi - c)
    float2 r;
    asm("{\n .reg .b16 l, h;\n mov.b32 {l, h}, %2;\n sub.rn.f32.bf16 %0, l, %3;\n sub.rn.f32.bf16 %1, h, %3;\n}\n"
        : "=f"(r.x), "=f"(r.y)
        : "r"(w), "f"(c));
    return r;
}
__device__ __forceinline__ float2 bf2_add(uint32_t w, float c) {  // (lo + c, hi + c)
    float2 r;
    asm("{\n .reg .b16 l, h;\n mov.b32 {l, h}, %2;\n add.rn.f32.bf16 %0, l, %3;\n add.rn.f32.bf16 %1, h, %3;\n}\n"
        : "=f"(r.x), "=f"(r.y)
        : "r"(w), "f"(c));
    return r;
}
__device__ __forceinline__ float2 bf2_fma(uint32_t a, uint32_t b, float2 c) {  // (a.lo*b.lo + c.x, a.hi*b.hi + c.y)
    float2 r;
    asm("{\n .reg .b16 al, ah, bl, bh;\n mov.b32 {al, ah}, %2;\n mov.b32 {bl, bh}, %3;\n"
        " fma.rn.f32.bf16 %0, al, bl, %4;\n fma.rn.f32.bf16 %1, ah, bh, %5;\n}\n"
        : "=f"(r.x), "=f"(r.y)
        : "r"(a), "r"(b), "f"(c.x), "f"(c.y));
    return r;
}

// Round two floats to a packed bf16 pair (RNE), like __floats2bfloat162_rn.
__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}

__device__ __forceinline__ void unpack8(const Vec8 &v, float (&f)[8]) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        f[2 * i] = bf_lo(v.w[i]);
        f[2 * i + 1] = bf_hi(v.w[i]);
    }
}

__device__ __forceinline__ Vec8 pack8(const float (&f)[8]) {
    Vec8 v;
#pragma unroll
    for (int i = 0; i < 4; ++i) v.w[i] = pack_bf2(f[2 * i], f[2 * i + 1]);
    return v;
}

__device__ __forceinline__ float bf16_round(float f) {
    return __bfloat162float(__float2bfloat16_rn(f));
}

// Position of unit i in a [rows, per_row] grid and the row's phase row % P (the table
// row), advanced by the grid stride without divisions: the stride's quotient, remainder
// and quotient mod P are taken once per thread.
struct UnitCursor {
    int64_t row, drow;
    uint32_t rem, drem, ph, dph;
    __device__ __forceinline__ UnitCursor(int64_t i, int64_t stride, uint32_t per_row, uint32_t P) {
        row = i / per_row;
        rem = (uint32_t)(i - row * per_row);
        ph = (uint32_t)(row % P);
        drow = stride / per_row;
        drem = (uint32_t)(stride - drow * per_row);
        dph = (uint32_t)(drow % P);
    }
    __device__ __forceinline__ void advance(uint32_t per_row, uint32_t P) {
        row += drow;
        rem += drem;
        ph += dph;
        if (rem >= per_row) {
            rem -= per_row;
            ++row;
            ++ph;
        }
        if (ph >= P) ph -= P;  // ph + dph + 1 < 2P
    }
};

// ------------------------------------------------- reference reduction replay
//
// The reference reduces a row of D2 = D/2 bf16 pairs with one CTA of T = D2 threads
// (D2 <= 1024 and a multiple of 32): thread t owns pair t, each warp reduces its 32
// values with __shfl_down_sync offsets 16,8,4,2,1 (cuda_utils.cuh:46-50), warp 0 then
// reduces the per-warp results the same way, padded with zeros to 32
// (layer_norm.cu:7-19, rms_norm.cu:40-53). Floating-point addition is commutative but
// not associative, so matching its bits means matching that tree.
//
// Here a row is owned by a "team" of LPR lanes (8, 16 or 32) of one warp. Lane l of the
// team holds chunks c = l + LPR*k (k < K) of 8 elements, i.e. pairs p = 4c + j (j < 4).
// Reference thread p sits in reference warp w = c/8 at reference lane r = 4(c%8) + j.
// So reference offsets 16/8/4 are lane XORs 4/2/1 inside the team (c%8 = l%8 since
// LPR % 8 == 0), and offsets 2/1 pair up j inside one lane. The warp-level tree runs as
// a transposed butterfly: at each lane-XOR step a lane keeps half of its k values and
// ships the other half to its partner, so K=8 costs 16+8+4 shuffles instead of 96.
// After it, lane l holds the sum of reference warp w = (l>>3) + (LPR/8)*k*(l), and the
// second-level tree over w maps each reference offset onto one more lane XOR.

template <int N>
struct Log2 {
    static constexpr int value = 1 + Log2<N / 2>::value;
};
template <>
struct Log2<1> {
    static constexpr int value = 0;
};

// One lane-XOR step of the warp-level tree over values cur[M][4] (M = live k values).
template <int M>
struct TreeStep {
    static constexpr int OUT = M > 1 ? M / 2 : 1;
    __device__ __forceinline__ static void run(const float (&cur)[M][4], float (&nxt)[OUT][4],
                                               int bit, int l, unsigned mask) {
        if constexpr (M > 1) {
            const bool upper = (l >> bit) & 1;
#pragma unroll
            for (int i = 0; i < M / 2; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float keep = upper ? cur[i + M / 2][j] : cur[i][j];
                    float send = upper ? cur[i][j] : cur[i + M / 2][j];
                    nxt[i][j] = keep + __shfl_xor_sync(mask, send, 1 << bit);
                }
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j)
                nxt[0][j] = cur[0][j] + __shfl_xor_sync(mask, cur[0][j], 1 << bit);
        }
    }
};

// Full reference block sum of the row's pair values v[k][j]; every lane of the team
// receives the result. LPR in {8,16,32}, K in {1,2,4,8}, D = 8*LPR*K <= 2048.
template <int LPR, int K>
__device__ __forceinline__ float ref_pair_tree_sum(const float (&v)[K][4], int l, unsigned mask) {
    static_assert(LPR == 8 || LPR == 16 || LPR == 32, "team size");
    static_assert(K == 1 || K == 2 || K == 4 || K == 8, "chunks per lane");
    constexpr int M1 = TreeStep<K>::OUT;
    constexpr int M2 = TreeStep<M1>::OUT;
    constexpr int M3 = TreeStep<M2>::OUT;
    float a[M1][4], b[M2][4], c[M3][4];
    TreeStep<K>::run(v, a, 2, l, mask);   // reference offset 16
    TreeStep<M1>::run(a, b, 1, l, mask);  // reference offset 8
    TreeStep<M2>::run(b, c, 0, l, mask);  // reference offset 4
    // reference offsets 2 and 1: pairs j^2, then j^1, inside the lane
    float s = (c[0][0] + c[0][2]) + (c[0][1] + c[0][3]);

    // Second level: reference warp 0 over w = (l>>3) + G*kstar, zero-padded to 32.
    constexpr int LG_G = Log2<LPR / 8>::value;
    constexpr int LG_K = Log2<K>::value;
    constexpr int NW = (LPR / 8) * K;  // reference warps in the row
#pragma unroll
    for (int i = 4; i >= 0; --i) {
        if ((1 << i) >= NW) continue;  // partner slot holds a padding zero: x + 0 == x
        const int lane_bit = i < LG_G ? 3 + i : (i - LG_G) + 3 - LG_K;
        s = s + __shfl_xor_sync(mask, s, 1 << lane_bit);
    }
    return s;
}

// The reference's CTA reduction itself (warp shfl_down tree, then warp 0 over the
// per-warp sums), for the generic one-CTA-per-row kernels. `red` holds >= 32 floats.
// Returns the total to every thread. Contains __syncthreads.
__device__ __forceinline__ float ref_cta_sum(float v, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nwarps = (blockDim.x + 31) >> 5;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_down_sync(0xffffffffu, v, off);
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = lane < nwarps ? red[lane] : 0.0f;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v += __shfl_down_sync(0xffffffffu, v, off);
        if (lane == 0) red[32] = v;
    }
    __syncthreads();
    float total = red[32];
    __syncthreads();  // red may be reused by the caller's next reduction
    return total;
}

// Block size the reference launchers use for a row of D elements (rms_norm.cu:126-128).
__host__ __device__ __forceinline__ int ref_row_threads(int D) {
    int D2 = D / 2;
    int t = (D2 <= 1024) ? ((D2 + 31) / 32 * 32) : 1024;
    return t < 32 ? 32 : t;
}

// ------------------------------------------------- programmatic dependent launch
// Every kernel is launched with programmatic stream serialisation, so its CTAs may be
// scheduled while the previous kernel in the stream drains. pdl_wait() -- the first
// statement of every kernel, before any global memory access -- blocks until that
// previous kernel has completed and its writes are visible (a no-op when the launch had
// no predecessor or was not programmatic). pdl_launch() lets the next kernel start its
// launch early; a CTA that exits counts as having called it.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------------------ host side

// Number of SMs of the current device (cached per device ordinal).
int sm_count();

// Bounded device waits of the elementwise table kernel that ran out on the current device
// (elementwise.cu; cleared when reset != 0). anima_wait_timeouts reports them with the
// channel norm's.
int ew_wait_timeouts(unsigned int *count, int reset);

// Raises a kernel's dynamic shared-memory limit to `bytes` on the current device, once
// per (device, slot); `slot` names the kernel (0..63). Returns ANIMA_OK or a cudaError_t.
int allow_dynamic_smem(const void *kernel, int bytes, int slot);

// Resident CTAs per SM of `kernel` launched with `block` threads and `smem` bytes of
// dynamic shared memory on the current device, raising the kernel's dynamic shared-memory
// limit first when smem > 48 KB. Cached per (device, kernel, smem). On failure returns 0
// and stores the status in *err.
int resident_ctas(const void *kernel, int block, int smem, int *err);

// CTAs for a grid-stride kernel: enough for `work` items at one per thread, but at most one
// resident wave (SMs x the CTAs of `kernel` that fit on one SM together), so no CTA waits
// for a second wave. On failure returns 0 and stores the status in *err.
unsigned wave_grid(const void *kernel, int block, int smem, int64_t work, int *err);

__host__ __device__ inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool aligned_to(const void *p, unsigned a) {
    return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

// True when [a, a+na) and [b, b+nb) overlap without being the same buffer start.
inline bool partial_overlap(const void *a, int64_t na, const void *b, int64_t nb) {
    uintptr_t x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
    if (x == y) return false;
    return x < y + (uintptr_t)nb && y < x + (uintptr_t)na;
}

// True when [a, a+na) and [b, b+nb) share any byte (the same start included).
inline bool overlaps(const void *a, int64_t na, const void *b, int64_t nb) {
    uintptr_t x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
    return x < y + (uintptr_t)nb && y < x + (uintptr_t)na;
}

// Launches `kernel` on `stream` with programmatic dependent launch allowed.
template <typename... KArgs, typename... Args>
inline void launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                   Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// The same, for a grid of thread-block clusters of `cluster` CTAs along x.
template <typename... KArgs, typename... Args>
inline void launch_cluster(void (*kernel)(KArgs...), unsigned cluster, dim3 grid, dim3 block, size_t smem,
                           cudaStream_t stream, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Status of the launch just issued (launch-configuration errors only; kernels run async).
inline int launch_status() {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ANIMA_OK : (int)e;
}

}  // namespace anima
