// rownorm.cu -- LayerNorm / adaLN / residual-gate adaLN / RMSNorm row kernels (sm_100a).
//
// Fast path (D a multiple of 64, D <= 2048, 16-byte aligned rows): the "segment"
// kernels below. Each lane owns one 64-element segment of a row -- the 32 pairs that
// one warp of the reference's row CTA reduces -- so the reference's addition tree is
// replayed exactly: its warp-level shfl_down tree as 31 in-register adds, its cross-warp
// level as lane XORs inside the row's team. Rows stream through a per-warp ring of
// shared-memory slots filled ahead by cp.async, and results leave through the same slot
// with coalesced 16-byte stores: every row is read from HBM once and written once (the
// reference reads it twice and runs three __syncthreads per reduction on a 1024-thread
// CTA per row). Outputs match the reference kernels bit for bit.
//
// Generic path (any even D, any 2-byte alignment): one CTA per row with the reference's
// own thread layout and scalar accesses. Same bits, reference-like speed.
#include "common.cuh"

namespace anima {
namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kRowBlock = 256;

// var = sum_sq/D - mean*mean: nvcc contracts the reference's expression
// (layer_norm.cu:49,107,179) into one fma.
__device__ __forceinline__ float ln_var(float sq, float mean, int D) {
    return fmaf(-mean, mean, __fdiv_rn(sq, (float)D));
}
// The same for the segment kernels, whose D = 64 * NW is a power of two.
template <int D>
__device__ __forceinline__ float ln_var_p2(float sq, float mean) {
    return fmaf(-mean, mean, div_pow2<D>(sq));
}

// sum_sq += h0*h0 + h1*h1 on unrounded fp32 h (layer_norm.cu:176): nvcc folds the first
// product into an fma with the second.
__device__ __forceinline__ float resid_sq_pair(float h0, float h1) { return fmaf(h0, h0, h1 * h1); }

// adaLN-Zero modulation folded into a norm: the reference adds the timestep embedding to the
// modulation vector in place (add_bf16(mod, temb, mod, 3D), transformer.cpp:407) before the
// norm reads shift and scale from it, then copies the gate out (:424). The *_temb entry points
// read mod and temb directly: each modulation value is bf16(float(mod) + float(temb)), the
// add_bf16 rounding (elementwise.cu:49-52), and CTA 0 writes this set's gate to gate_out.
struct TembFold {
    const anima_bf16 *tsc = nullptr, *tsh = nullptr;  // temb slices added to scale and shift
    const anima_bf16 *gmod = nullptr, *gtemb = nullptr;  // this set's gate: mod and temb slices
    anima_bf16 *gate_out = nullptr;                       // nullptr: no fold
};

__device__ __forceinline__ float bf16_add(float a, float b) { return bf16_round(a + b); }

// gate_out[d] = bf16(mod_gate[d] + temb_gate[d]) for d < D, spread over the whole grid (at
// most one 16-byte chunk or one element per thread, so it costs one memory round trip).
__device__ __forceinline__ void fold_gate(const TembFold &t, int D) {
    if (!t.gate_out) return;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t nthr = (int64_t)gridDim.x * blockDim.x;
    if (aligned16(t.gmod) && aligned16(t.gtemb) && aligned16(t.gate_out) && D % 8 == 0) {
        for (int64_t c = tid; c < D / 8; c += nthr) {
            float a[8], b[8];
            unpack8(ld_cached(t.gmod + 8 * c), a);
            unpack8(ld_cached(t.gtemb + 8 * c), b);
#pragma unroll
            for (int e = 0; e < 8; ++e) a[e] = bf16_add(a[e], b[e]);
            st_vec(t.gate_out + 8 * c, pack8(a));
        }
    } else {
        for (int64_t d = tid; d < D; d += nthr) {
            const float g = bf16_add(__bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(t.gmod)[d]),
                                     __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(t.gtemb)[d]));
            reinterpret_cast<__nv_bfloat16 *>(t.gate_out)[d] = __float2bfloat16_rn(g);
        }
    }
}

// ------------------------------------------------ segment kernels (fast path)
//
// A row of D elements (D % 64 == 0, D <= 2048) is NW = D/64 "segments" of 64 elements:
// exactly the 32 pairs one reference warp reduces (thread t owns pair t, so warp w owns
// elements 64w..64w+63). Each lane owns one segment, so the reference's warp-level
// shfl_down tree becomes 31 in-register adds in the same order, and its cross-warp
// level is log2(NW) lane XORs inside the row's team of NW lanes. A warp therefore
// handles a 4 KB "unit" of G = 32/NW consecutive rows per input.
//
// Data movement: persistent CTAs of 4 warps; each warp owns a ring of NST unit slots in
// shared memory. Units are copied in NST ahead with 16-byte cp.async (coalesced: lane l
// copies chunks l, l+32, ...), read back per segment, the outputs are written into the
// same slot and stored to global memory coalesced again. Slots are XOR-swizzled at
// 16-byte granularity inside each 128-byte group so that both patterns are free of bank
// conflicts. Broadcast vectors (scale, shift, gate, weight) are staged once per CTA in shared
// memory as bf16 chunks, swizzled the same way, and converted as they are read.

constexpr int kUnitChunks = 256;  // 16-byte chunks per input per unit (4 KB)

__device__ __forceinline__ int swz(int c) { return (c & ~7) | ((c & 7) ^ ((c >> 3) & 7)); }

// CTA size, ring depth and occupancy target: 4 warps with 2 slots each; one-input ops run 4
// CTAs per SM (at most 128 registers per thread), two- and three-input ops 2.
template <int NIN>
struct SegShape {
    static constexpr int kWarps = 4;
    static constexpr int kThreads = kWarps * 32;
    static constexpr int kStages = 2;
    static constexpr int kMinCtas = NIN == 1 ? 4 : 2;
    static constexpr int kRingBytes = kWarps * kStages * NIN * kUnitChunks * 16;
};

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const unsigned a = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(a), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// The reference warp's shfl_down tree over the 32 pairs of one segment, in registers, as
// packed fp32x2 adds (each lane of FADD2 rounds like the scalar add, so the sums are the
// reference's bit for bit at half the instructions). q(k, h) returns pairs 4k+2h and
// 4k+2h+1 (chunk k, words 2h and 2h+1). With scalar a_s[4k+2h+t] = a[2k+h].t, each level
// below adds exactly the pairs the reference's offset adds.
template <class PairFn2>
__device__ __forceinline__ float seg_tree(PairFn2 q) {
    float2 a[8], b[4], c[2];
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int h = 0; h < 2; ++h) a[2 * k + h] = __fadd2_rn(q(k, h), q(k + 4, h));  // offset 16
#pragma unroll
    for (int i = 0; i < 4; ++i) b[i] = __fadd2_rn(a[i], a[i + 4]);                    // offset 8
#pragma unroll
    for (int i = 0; i < 2; ++i) c[i] = __fadd2_rn(b[i], b[i + 2]);                    // offset 4
    const float2 d = __fadd2_rn(c[0], c[1]);                                           // offset 2
    return d.x + d.y;                                                                  // offset 1
}

// Words 2h, 2h+1 of a chunk as (low elements) and (high elements).
__device__ __forceinline__ float2 lo2(const Vec8 &v, int h) { return make_float2(bf_lo(v.w[2 * h]), bf_lo(v.w[2 * h + 1])); }
__device__ __forceinline__ float2 hi2(const Vec8 &v, int h) { return make_float2(bf_hi(v.w[2 * h]), bf_hi(v.w[2 * h + 1])); }

// Pair sums of squares fmaf(b, b, a*a) (nvcc's contraction of the reference's a*a + b*b).
__device__ __forceinline__ float2 sq_pairs(const Vec8 &v, int h) {
    const float2 a = lo2(v, h), b = hi2(v, h);
    return __ffma2_rn(b, b, __fmul2_rn(a, a));
}

// The reference's second level: warp 0 reduces the NW per-warp sums, zero-padded to 32.
// Segment s sits in lane s of the row's team, so reference offset o is lane XOR o.
template <int NW>
__device__ __forceinline__ float seg_cross(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
        if (off < NW) v = v + __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

// Sum and sum of squares of a plain bf16 segment (pair values: v0+v1, round(v0^2+v1^2)).
__device__ __forceinline__ void seg_stats(const Vec8 (&v)[8], float &sum, float &sq) {
    sum = seg_tree([&](int k, int h) { return __fadd2_rn(lo2(v[k], h), hi2(v[k], h)); });
    sq = seg_tree([&](int k, int h) { return sq_pairs(v[k], h); });
}

__device__ __forceinline__ void load_seg(const Vec8 *buf, int lane, Vec8 (&v)[8]) {
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = buf[swz(8 * lane + k)];
}

// Broadcast vector b of an op, chunk k of segment `seg`, as 8 floats: the vectors are staged
// as bf16 chunks in the rows' swizzled layout (vector b starts D/8 chunks after vector b-1);
// `plus1` adds the reference's 1.0f (its (1.0f + scale[d]) in fp32) here.
__device__ __forceinline__ void bvec8(const float *bc, int b, int D, int seg, int k, bool plus1, float (&f)[8]) {
    unpack8(reinterpret_cast<const Vec8 *>(bc)[b * (D >> 3) + swz(8 * seg + k)], f);
    if (plus1) {
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
            const float2 t = __fadd2_rn(make_float2(f[e], f[e + 1]), make_float2(1.0f, 1.0f));
            f[e] = t.x;
            f[e + 1] = t.y;
        }
    }
}

// Packed fp32x2 arithmetic (sm_100 FFMA2/FADD2/FMUL2): two lanes of IEEE round-to-nearest
// per instruction, so results equal the scalar ops bit for bit at half the issue cost.
__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }

// The adaLN modulation on packed bf16 words: out = fma((x - mean) * inv, 1 + scale, shift),
// rounded to bf16 (the normalised value rounded to bf16 first for kRoundFirst; nvcc contracts
// the reference's n * (1.0f + scale) + shift into this fma, layer_norm.cu:121-122,192-193); x - mean and
// 1 + scale by the mixed-precision ops above, in the reference's fp32 roundings.
template <bool kRoundFirst>
__device__ __forceinline__ Vec8 ln_modulate_w(const Vec8 &x, float mean, float inv, const Vec8 &scale,
                                              const Vec8 &shift) {
    Vec8 o;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float2 n = __fmul2_rn(bf2_sub(x.w[j], mean), f2(inv, inv));
        if constexpr (kRoundFirst) n = f2(bf16_round(n.x), bf16_round(n.y));
        const float2 r = __ffma2_rn(n, bf2_add(scale.w[j], 1.0f), f2(bf_lo(shift.w[j]), bf_hi(shift.w[j])));
        o.w[j] = pack_bf2(r.x, r.y);
    }
    return o;
}

// Broadcast vector b's staged bf16 chunk k of segment `seg` (the layout bvec8 reads).
__device__ __forceinline__ const Vec8 &bchunk(const float *bc, int b, int D, int seg, int k) {
    return reinterpret_cast<const Vec8 *>(bc)[b * (D >> 3) + swz(8 * seg + k)];
}

__device__ __forceinline__ float bf(const anima_bf16 *p, int i) {
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[i]);
}

// ---- ops: NIN streamed inputs, NOUT outputs (written over input buffers 0..NOUT-1),
// NB broadcast vectors (bf16 in shared memory, read through bvec8).

struct LayerNormOp {  // layer_norm.cu:26-59
    static constexpr int NIN = 1, NOUT = 1, NB = 0;
    const anima_bf16 *x;
    anima_bf16 *out;
    float eps;
    __device__ const anima_bf16 *src(int) const { return x; }
    __device__ anima_bf16 *dst(int) const { return out; }
    template <int NW>
    __device__ void segment(Vec8 *slot, const float *, int lane, int, int D) const {
        Vec8 v[8];
        load_seg(slot, lane, v);
        float sum, sq;
        seg_stats(v, sum, sq);
        sum = seg_cross<NW>(sum);
        sq = seg_cross<NW>(sq);
        const float mean = div_pow2<64 * NW>(sum);
        const float inv = rsqrtf(ln_var_p2<64 * NW>(sq, mean) + eps);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            Vec8 o;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 n = __fmul2_rn(bf2_sub(v[k].w[j], mean), f2(inv, inv));
                o.w[j] = pack_bf2(n.x, n.y);
            }
            slot[swz(8 * lane + k)] = o;
        }
    }
};

// kRoundFirst false: adaLN (layer_norm.cu:83-125); true: LN -> bf16 -> modulate.
// kTemb: the adaLN-Zero modulation fold (TembFold) is applied.
template <bool kRoundFirst, bool kTemb = false>
struct AdaLNOp {
    static constexpr int NIN = 1, NOUT = 1, NB = 2;
    const anima_bf16 *x, *scale, *shift;
    anima_bf16 *out;
    float eps;
    __device__ const anima_bf16 *src(int) const { return x; }
    __device__ anima_bf16 *dst(int) const { return out; }
    TembFold fold = {};
    static constexpr bool kFold = kTemb;
    __device__ const anima_bf16 *bvec(int i) const { return i == 0 ? scale : shift; }
    __device__ const anima_bf16 *btemb(int i) const { return i == 0 ? fold.tsc : fold.tsh; }
    template <int NW>
    __device__ void segment(Vec8 *slot, const float *bc, int lane, int seg, int D) const {
        Vec8 v[8];
        load_seg(slot, lane, v);
        float sum, sq;
        seg_stats(v, sum, sq);
        sum = seg_cross<NW>(sum);
        sq = seg_cross<NW>(sq);
        const float mean = div_pow2<64 * NW>(sum);
        const float inv = rsqrtf(ln_var_p2<64 * NW>(sq, mean) + eps);
#pragma unroll
        for (int k = 0; k < 8; ++k)
            slot[swz(8 * lane + k)] =
                ln_modulate_w<kRoundFirst>(v[k], mean, inv, bchunk(bc, 0, D, seg, k), bchunk(bc, 1, D, seg, k));
    }
};

template <bool kTemb = false>
struct ResGateAdaLNOp {  // layer_norm.cu:146-196
    static constexpr int NIN = 2, NOUT = 2, NB = 3;
    anima_bf16 *hidden;
    const anima_bf16 *sub_out, *gate, *scale, *shift;
    anima_bf16 *normed;
    float eps;
    __device__ const anima_bf16 *src(int i) const { return i == 0 ? hidden : sub_out; }
    __device__ anima_bf16 *dst(int o) const { return o == 0 ? hidden : normed; }
    TembFold fold = {};  // the gate is the previous set's, already summed
    static constexpr bool kFold = kTemb;
    __device__ const anima_bf16 *bvec(int i) const { return i == 0 ? gate : (i == 1 ? scale : shift); }
    __device__ const anima_bf16 *btemb(int i) const { return i == 0 ? nullptr : (i == 1 ? fold.tsc : fold.tsh); }
    template <int NW>
    __device__ void segment(Vec8 *slot, const float *bc, int lane, int seg, int D) const {
        Vec8 x[8], y[8];
        load_seg(slot, lane, x);
        load_seg(slot + kUnitChunks, lane, y);
        // h = x + y*gate in fp32 (the bf16 product is exact, so fma rounds like the
        // reference); the statistics use the unrounded h, the output the bf16 h.
        float h[8][8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const Vec8 &g = bchunk(bc, 0, D, seg, k);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 hv = bf2_fma(y[k].w[j], g.w[j], f2(bf_lo(x[k].w[j]), bf_hi(x[k].w[j])));
                h[k][2 * j] = hv.x;
                h[k][2 * j + 1] = hv.y;
            }
        }
        // pairs (h[k][4i], h[k][4i+1]) and (h[k][4i+2], h[k][4i+3]); resid_sq_pair packed
        float sum = seg_tree([&](int k, int i) {
            return __fadd2_rn(f2(h[k][4 * i], h[k][4 * i + 2]), f2(h[k][4 * i + 1], h[k][4 * i + 3]));
        });
        float sq = seg_tree([&](int k, int i) {
            const float2 h0 = f2(h[k][4 * i], h[k][4 * i + 2]), h1 = f2(h[k][4 * i + 1], h[k][4 * i + 3]);
            return __ffma2_rn(h0, h0, __fmul2_rn(h1, h1));
        });
        sum = seg_cross<NW>(sum);
        sq = seg_cross<NW>(sq);
        const float mean = div_pow2<64 * NW>(sum);
        const float inv = rsqrtf(ln_var_p2<64 * NW>(sq, mean) + eps);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const Vec8 hb = pack8(h[k]);
            slot[swz(8 * lane + k)] = hb;
            slot[kUnitChunks + swz(8 * lane + k)] =
                ln_modulate_w<false>(hb, mean, inv, bchunk(bc, 1, D, seg, k), bchunk(bc, 2, D, seg, k));
        }
    }
};

template <bool kWeight>
struct RmsOp {  // rms_norm.cu:9-67
    static constexpr int NIN = 1, NOUT = 1, NB = kWeight ? 1 : 0;
    const anima_bf16 *x, *weight;
    anima_bf16 *out;
    float eps;
    __device__ const anima_bf16 *src(int) const { return x; }
    __device__ anima_bf16 *dst(int) const { return out; }
    TembFold fold = {};
    static constexpr bool kFold = false;
    __device__ const anima_bf16 *bvec(int) const { return weight; }
    __device__ const anima_bf16 *btemb(int) const { return nullptr; }
    template <int NW>
    __device__ void segment(Vec8 *slot, const float *bc, int lane, int seg, int D) const {
        Vec8 v[8];
        load_seg(slot, lane, v);
        float sq = seg_tree([&](int k, int h) { return sq_pairs(v[k], h); });
        sq = seg_cross<NW>(sq);
        const float r = rsqrtf(div_pow2<64 * NW>(sq) + eps);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            float f[8];
            unpack8(v[k], f);
            if constexpr (kWeight) {
                float w[8];
                bvec8(bc, 0, D, seg, k, false, w);
#pragma unroll
                for (int e = 0; e < 8; e += 2) {
                    const float2 o = __fmul2_rn(__fmul2_rn(f2(f[e], f[e + 1]), f2(r, r)), f2(w[e], w[e + 1]));
                    f[e] = o.x;
                    f[e + 1] = o.y;
                }
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) f[e] = f[e] * r;
            }
            slot[swz(8 * lane + k)] = pack8(f);
        }
    }
};

struct AdaRmsOp {  // adaln.cu:11-58 (per-row scale/shift streamed alongside x)
    static constexpr int NIN = 3, NOUT = 1, NB = 0;
    const anima_bf16 *x, *scale, *shift;
    anima_bf16 *out;
    float eps;
    __device__ const anima_bf16 *src(int i) const { return i == 0 ? x : (i == 1 ? scale : shift); }
    __device__ anima_bf16 *dst(int) const { return out; }
    template <int NW>
    __device__ void segment(Vec8 *slot, const float *, int lane, int, int D) const {
        Vec8 v[8];
        load_seg(slot, lane, v);
        float sq = seg_tree([&](int k, int h) { return sq_pairs(v[k], h); });
        sq = seg_cross<NW>(sq);
        const float r = rsqrtf(div_pow2<64 * NW>(sq) + eps);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            float f[8], sc[8], sh[8];
            unpack8(v[k], f);
            unpack8(slot[kUnitChunks + swz(8 * lane + k)], sc);
            unpack8(slot[2 * kUnitChunks + swz(8 * lane + k)], sh);
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = fmaf(f[e] * r, 1.0f + sc[e], sh[e]);
            slot[swz(8 * lane + k)] = pack8(f);
        }
    }
};

// The temb-fold ops' broadcast vectors (modulation + temb, rounded to bf16 as add_bf16 stores
// them) -> bf16 chunks in shared memory, in the rows' swizzled layout. Split in two so that the
// row prefetch can be issued in between: the vectors' 16-byte loads go out first (they hit L2
// and must not queue behind megabytes of rows), then the rows, then the sums. Vectors that are
// not 16-byte aligned are read with scalar loads in the second half. (The other ops copy their
// vectors with cp.async; see row_seg.)
template <class Op>
struct BcastStage {
    static constexpr int kThreads = SegShape<Op::NIN>::kThreads;
    static constexpr int kPer = (Op::NB * 256 + kThreads - 1) / kThreads;  // D <= 2048: <= 256 chunks per vector
    Vec8 v[kPer], t[kPer];

    __device__ __forceinline__ void load(const Op &op, int D) {
        const int nch = D >> 3;
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const int i = threadIdx.x + k * kThreads;
            if (i < Op::NB * nch) {
                const int b = i / nch;
                const anima_bf16 *src = op.bvec(b), *add = Op::kFold ? op.btemb(b) : nullptr;
                if (aligned16(src) && (!add || aligned16(add))) {
                    v[k] = ld_cached(src + 8 * (i - b * nch));
                    if (add) t[k] = ld_cached(add + 8 * (i - b * nch));
                }
            }
        }
    }
    __device__ __forceinline__ void store(const Op &op, float *bc, int D) const {
        const int nch = D >> 3;
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const int i = threadIdx.x + k * kThreads;
            if (i < Op::NB * nch) {
                const int b = i / nch, c = i - b * nch;
                const anima_bf16 *src = op.bvec(b), *add = Op::kFold ? op.btemb(b) : nullptr;
                float f[8];
                if (aligned16(src) && (!add || aligned16(add))) {
                    unpack8(v[k], f);
                    if (add) {
                        float g[8];
                        unpack8(t[k], g);
#pragma unroll
                        for (int e = 0; e < 8; ++e) f[e] = bf16_add(f[e], g[e]);
                    }
                } else {
#pragma unroll
                    for (int e = 0; e < 8; ++e) f[e] = add ? bf16_add(bf(src, 8 * c + e), bf(add, 8 * c + e)) : bf(src, 8 * c + e);
                }
                // bf16 chunks in the rows' swizzled layout (the values are bf16 already, so the
                // packing is exact); the reference's 1.0f is added where they are read
                reinterpret_cast<Vec8 *>(bc)[b * nch + swz(c)] = pack8(f);
            }
        }
    }
};

// Bytes per broadcast-vector element in shared memory (bf16 staging).
template <class Op>
__host__ __device__ constexpr int bc_bytes() { return 2; }

// Whether the op folds temb into its broadcast vectors (ops without vectors have no kFold).
template <class Op>
__host__ __device__ constexpr bool op_folds() {
    if constexpr (Op::NB > 0) return Op::kFold;
    return false;
}

template <int NW, class Op>
__global__ void __launch_bounds__(SegShape<Op::NIN>::kThreads, SegShape<Op::NIN>::kMinCtas)
    row_seg(Op op, int64_t N, int D) {
    pdl_wait();
    constexpr int NIN = Op::NIN, NOUT = Op::NOUT, NB = Op::NB;
    constexpr int G = 32 / NW;  // rows per unit
    constexpr int NST = SegShape<NIN>::kStages;
    constexpr int kSegWarps = SegShape<NIN>::kWarps;
    constexpr int kRowChunks = NW * 8;
    extern __shared__ __align__(16) unsigned char seg_smem[];
    float *bc = reinterpret_cast<float *>(seg_smem);
    Vec8 *ring = reinterpret_cast<Vec8 *>(seg_smem + (size_t)NB * D * bc_bytes<Op>()) +
                 (size_t)(threadIdx.x >> 5) * NST * NIN * kUnitChunks;
    const int lane = threadIdx.x & 31;
    const int64_t units = (N + G - 1) / G;
    const int64_t nwarps = (int64_t)gridDim.x * kSegWarps;
    const int64_t first = (int64_t)blockIdx.x * kSegWarps + (threadIdx.x >> 5);
    auto unit_chunks = [&](int64_t u) {
        const int64_t left = N - u * G;
        return left >= G ? kUnitChunks : (int)left * kRowChunks;
    };
    auto copy_unit = [&](int64_t u, int st) {
        if (u < units) {
            const int nch = unit_chunks(u);
#pragma unroll
            for (int in = 0; in < NIN; ++in) {
                const anima_bf16 *src = op.src(in) + u * G * (int64_t)D;
                Vec8 *buf = ring + (st * NIN + in) * kUnitChunks;
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const int c = lane + 32 * k;
                    if (c < nch) cp_async16(buf + swz(c), src + (int64_t)c * 8);
                }
            }
        }
    };
    auto issue = [&](int64_t u, int st) {
        copy_unit(u, st);
        cp_async_commit();  // one group per unit, empty or not, keeps the counting uniform
    };
    if constexpr (NB > 0 && !op_folds<Op>()) {
        // the vectors as bf16 chunks, swizzled like a unit, in the same copy group as the first
        // unit: no conversion pass, and half the shared-memory reads per row of an fp32 stage.
        // The unit's copies go first, so the rows' DRAM reads queue ahead of the vectors' L2
        // reads, which every CTA makes at once (at 4096 x 2048: adaLN 8.59 -> 8.18 us,
        // RMSNorm 7.71 -> 7.11, residual gate + adaLN 14.15 -> 13.18).
        copy_unit(first, 0);
        const int nch = D >> 3;
        Vec8 *bcv = reinterpret_cast<Vec8 *>(seg_smem);
        for (int i = threadIdx.x; i < NB * nch; i += SegShape<NIN>::kThreads) {
            const int b = i / nch, c = i - b * nch;
            cp_async16(bcv + b * nch + swz(c), op.bvec(b) + 8 * c);
        }
        cp_async_commit();
#pragma unroll
        for (int st = 1; st < NST; ++st) issue(first + st * nwarps, st);
        cp_async_wait<NST - 1>();  // group 0 (this warp's first unit and the vectors) has landed ...
        __syncthreads();           // ... for every thread
    } else if constexpr (NB > 0) {
        // Here the vectors go first: they come through registers and are summed and stored
        // before the ring loop, so every warp waits on them; issued after the first unit they
        // cost 0.4-0.9 us per launch at 8192 x 2048.
        BcastStage<Op> bcs;
        bcs.load(op, D);
#pragma unroll
        for (int st = 0; st < NST; ++st) issue(first + st * nwarps, st);
        if constexpr (Op::kFold) fold_gate(op.fold, D);  // its loads overlap the vectors' and rows'
        bcs.store(op, bc, D);
        __syncthreads();
    } else {
#pragma unroll
        for (int st = 0; st < NST; ++st) issue(first + st * nwarps, st);
    }
    int st = 0;
    for (int64_t u = first; u < units; u += nwarps) {
        cp_async_wait<NST - 1>();  // this lane's copies of unit u have landed ...
        __syncwarp();              // ... and so have every other lane's
        Vec8 *slot = ring + st * NIN * kUnitChunks;
        op.template segment<NW>(slot, bc, lane, lane % NW, D);
        __syncwarp();
        const int nch = unit_chunks(u);
#pragma unroll
        for (int o = 0; o < NOUT; ++o) {
            anima_bf16 *dst = op.dst(o) + u * G * (int64_t)D;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int c = lane + 32 * k;
                if (c < nch) st_vec(dst + (int64_t)c * 8, slot[o * kUnitChunks + swz(c)]);
            }
        }
        __syncwarp();  // every lane is done with the slot before it is refilled
        issue(u + (int64_t)NST * nwarps, st);
        st = st + 1 == NST ? 0 : st + 1;
    }
    pdl_launch();
    cp_async_wait<0>();
}

// ------------------------------------------------ small-row RMSNorm (D <= 256)
// Per-head QK-norm rows (D = 128, 64) are a few hundred bytes, too short for the unit
// pipeline above to pay off. Here every 8-lane team loads its row with direct 16-byte
// loads, all K chunks issued at once: 32 rows per 256-thread CTA and up to 64 resident
// warps per SM, so a launch keeps most of its rows in flight together. The reference tree is replayed with the transposed butterfly of
// ref_pair_tree_sum (lanes hold chunks l and l+8k, i.e. reference lanes 4(l%8)+j).
template <int K, bool kWeight>
__global__ void __launch_bounds__(kRowBlock) rms_small(const anima_bf16 *x, const anima_bf16 *w, anima_bf16 *out,
                                                       int64_t N, int D, float eps) {
    pdl_wait();
    constexpr int LPR = 8;
    const int l = threadIdx.x & (LPR - 1);
    const int64_t row = (int64_t)blockIdx.x * (kRowBlock / LPR) + threadIdx.x / LPR;
    const bool live = row < N;
    const anima_bf16 *xr = x + row * (int64_t)D;
    Vec8 v[K], wv[K];
#pragma unroll
    for (int k = 0; k < K; ++k) v[k] = live ? ld_stream(xr + (l + LPR * k) * 8) : Vec8{{0u, 0u, 0u, 0u}};
    if constexpr (kWeight) {
#pragma unroll
        for (int k = 0; k < K; ++k) wv[k] = ld_cached(w + (l + LPR * k) * 8);
    }
    float q[K][4];
#pragma unroll
    for (int k = 0; k < K; ++k)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float a = bf_lo(v[k].w[j]), b = bf_hi(v[k].w[j]);
            q[k][j] = fmaf(b, b, a * a);
        }
    // Scalar squares and the division kept on purpose: packed squares (sq_pair2), squares on
    // the mixed-precision bf16 fma and the exact multiply by 1/D (div_pow2) each made this
    // load-latency-bound kernel slower (6.61 -> 6.80-6.84 us at [4096 x 16, 128]).
    const float r = rsqrtf(__fdiv_rn(ref_pair_tree_sum<LPR, K>(q, l, kFull), (float)D) + eps);
    pdl_launch();
    if (!live) return;
    anima_bf16 *o = out + row * (int64_t)D;
#pragma unroll
    for (int k = 0; k < K; ++k) {
        float f[8];
        unpack8(v[k], f);
        if constexpr (kWeight) {
            float g[8];
            unpack8(wv[k], g);
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
                const float2 t = __fmul2_rn(__fmul2_rn(f2(f[e], f[e + 1]), f2(r, r)), f2(g[e], g[e + 1]));
                f[e] = t.x;
                f[e + 1] = t.y;
            }
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = f[e] * r;
        }
        st_vec(o + (l + LPR * k) * 8, pack8(f));
    }
}

// ------------------------------------------- generic (reference-structured) kernels
// One CTA of ref_row_threads(D) threads per row, thread t owning pairs t, t+T, ...,
// scalar bf16 accesses (valid for any 2-byte alignment), reference reduction tree.

__device__ __forceinline__ float ldb(const anima_bf16 *p) {
    return __bfloat162float(*reinterpret_cast<const __nv_bfloat16 *>(p));
}
__device__ __forceinline__ void stb(anima_bf16 *p, float f) {
    *reinterpret_cast<__nv_bfloat16 *>(p) = __float2bfloat16_rn(f);
}

enum class GenKind { LayerNorm, AdaLN, LnModulate, Rms, AdaRms, ResGate };

struct GenArgs {
    const anima_bf16 *x;        // x, or hidden for ResGate
    anima_bf16 *hidden;         // ResGate only
    const anima_bf16 *y, *gate; // ResGate only
    const anima_bf16 *scale, *shift, *weight;
    anima_bf16 *out;
    int D;
    float eps;
    TembFold fold = {};
};

// scale[d] or shift[d], with the folded temb added when there is one.
__device__ __forceinline__ float modv(const anima_bf16 *v, const anima_bf16 *t, int d) {
    return t ? bf16_add(ldb(v + d), ldb(t + d)) : ldb(v + d);
}

template <GenKind KIND>
__global__ void row_generic(GenArgs a, int64_t N) {
    pdl_wait();
    fold_gate(a.fold, a.D);
    __shared__ float red[33];
    const int D2 = a.D / 2, T = blockDim.x;
    for (int64_t row = blockIdx.x; row < N; row += gridDim.x) {
        const int64_t base = row * (int64_t)a.D;
        float s = 0.0f, q = 0.0f;
        for (int i = threadIdx.x; i < D2; i += T) {
            const int64_t e = base + 2 * i;
            if constexpr (KIND == GenKind::ResGate) {
                float h0 = fmaf(ldb(a.y + e), ldb(a.gate + 2 * i), ldb(a.hidden + e));
                float h1 = fmaf(ldb(a.y + e + 1), ldb(a.gate + 2 * i + 1), ldb(a.hidden + e + 1));
                stb(a.hidden + e, h0);
                stb(a.hidden + e + 1, h1);
                s += h0 + h1;
                q += resid_sq_pair(h0, h1);
            } else if constexpr (KIND == GenKind::AdaLN) {
                float v0 = ldb(a.x + e), v1 = ldb(a.x + e + 1);
                s += v0 + v1;
                q += fmaf(v1, v1, v0 * v0);
            } else {  // layer_norm.cu:44-46 / rms_norm.cu:35-36: two chained fmas
                float v0 = ldb(a.x + e), v1 = ldb(a.x + e + 1);
                s += v0 + v1;
                q = fmaf(v0, v0, q);
                q = fmaf(v1, v1, q);
            }
        }
        constexpr bool kMean = KIND == GenKind::LayerNorm || KIND == GenKind::AdaLN ||
                               KIND == GenKind::LnModulate || KIND == GenKind::ResGate;
        float mean = 0.0f, inv;
        if constexpr (kMean) {
            mean = __fdiv_rn(ref_cta_sum(s, red), (float)a.D);
            inv = rsqrtf(ln_var(ref_cta_sum(q, red), mean, a.D) + a.eps);
        } else {
            inv = rsqrtf(__fdiv_rn(ref_cta_sum(q, red), (float)a.D) + a.eps);
        }
        // Pass 2 over the thread's own pairs, as in the reference (ResGate re-reads the
        // bf16 hidden it wrote in pass 1).
        for (int i = threadIdx.x; i < D2; i += T) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int d = 2 * i + h;
                const int64_t e = base + d;
                float o;
                if constexpr (KIND == GenKind::LayerNorm) {
                    o = (ldb(a.x + e) - mean) * inv;
                } else if constexpr (KIND == GenKind::AdaLN) {
                    o = fmaf((ldb(a.x + e) - mean) * inv, 1.0f + modv(a.scale, a.fold.tsc, d),
                             modv(a.shift, a.fold.tsh, d));
                } else if constexpr (KIND == GenKind::LnModulate) {
                    o = fmaf(bf16_round((ldb(a.x + e) - mean) * inv), 1.0f + ldb(a.scale + d),
                             ldb(a.shift + d));
                } else if constexpr (KIND == GenKind::ResGate) {
                    o = fmaf((ldb(a.hidden + e) - mean) * inv, 1.0f + modv(a.scale, a.fold.tsc, d),
                             modv(a.shift, a.fold.tsh, d));
                } else if constexpr (KIND == GenKind::Rms) {
                    o = ldb(a.x + e) * inv;
                    if (a.weight) o = o * ldb(a.weight + d);
                } else {  // AdaRms
                    o = fmaf(ldb(a.x + e) * inv, 1.0f + ldb(a.scale + e), ldb(a.shift + e));
                }
                stb(a.out + e, o);
            }
        }
    }
}

// gemma_ops.cu:132-168: scalar loop over D with min(roundup32(D),1024) threads per row.
__global__ void gemma_rms_generic(const anima_bf16 *x, const anima_bf16 *w, anima_bf16 *out,
                                  int64_t N, int D, float eps) {
    pdl_wait();
    __shared__ float red[33];
    for (int64_t row = blockIdx.x; row < N; row += gridDim.x) {
        const int64_t base = row * (int64_t)D;
        float q = 0.0f;
        for (int i = threadIdx.x; i < D; i += blockDim.x) {
            float v = ldb(x + base + i);
            q += v * v;
        }
        const float inv = rsqrtf(__fdiv_rn(ref_cta_sum(q, red), (float)D) + eps);
        for (int i = threadIdx.x; i < D; i += blockDim.x)
            stb(out + base + i, (ldb(x + base + i) * inv) * (1.0f + ldb(w + i)));
        __syncthreads();
    }
}

// ------------------------------------------------------------- dispatch

template <class Op, int NW>
int launch_seg(const Op &op, int64_t N, int D, cudaStream_t s) {
    const int smem = Op::NB * D * bc_bytes<Op>() + SegShape<Op::NIN>::kRingBytes;
    auto kern = row_seg<NW, Op>;
    int err = ANIMA_OK;
    constexpr int kSegWarps = SegShape<Op::NIN>::kWarps, kSegThreads = SegShape<Op::NIN>::kThreads;
    const int per_sm = resident_ctas((const void *)kern, kSegThreads, smem, &err);
    if (per_sm <= 0) return err != ANIMA_OK ? err : ANIMA_ERR_NO_DEVICE;
    constexpr int G = 32 / NW;
    const int64_t units = (N + G - 1) / G;
    int64_t grid = (units + kSegWarps - 1) / kSegWarps;
    const int64_t cap = (int64_t)per_sm * sm_count();
    if (grid > cap) grid = cap;
    launch(kern, (unsigned)grid, kSegThreads, (size_t)smem, s, op, N, D);
    return launch_status();
}

// Fast path for D in {64, 128, ..., 2048}: one 64-element segment per lane.
template <class Op>
bool dispatch_seg(const Op &op, int64_t N, int D, cudaStream_t s, int &status) {
    switch (D) {
    case 64: status = launch_seg<Op, 1>(op, N, D, s); return true;
    case 128: status = launch_seg<Op, 2>(op, N, D, s); return true;
    case 256: status = launch_seg<Op, 4>(op, N, D, s); return true;
    case 512: status = launch_seg<Op, 8>(op, N, D, s); return true;
    case 1024: status = launch_seg<Op, 16>(op, N, D, s); return true;
    case 2048: status = launch_seg<Op, 32>(op, N, D, s); return true;
    default: return false;
    }
}

inline unsigned generic_grid(int64_t N) { return (unsigned)(N < 2147483647 ? N : 2147483647); }

int check_row_args(int64_t N, int D) {
    if (N < 0 || D <= 0 || (D & 1)) return ANIMA_ERR_BAD_SHAPE;
    if (N > 0 && (int64_t)D > INT64_MAX / N) return ANIMA_ERR_TOO_LARGE;
    return ANIMA_OK;
}

bool bf16_ok(const void *p) { return aligned_to(p, 2); }

}  // namespace
}  // namespace anima

using namespace anima;

// ================================================================ C ABI

extern "C" int anima_layer_norm_bf16(const anima_bf16 *x, anima_bf16 *out, int N, int D, float eps,
                                     anima_stream_t stream) {
    if (int e = check_row_args(N, D)) return e;
    if (N == 0) return ANIMA_OK;
    if (!x || !out) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(x) || !bf16_ok(out)) return ANIMA_ERR_MISALIGNED;
    const int64_t n = (int64_t)N * D * 2;
    if (partial_overlap(x, n, out, n)) return ANIMA_ERR_OVERLAP;
    int st;
    if (aligned16(x) && aligned16(out) && dispatch_seg(LayerNormOp{x, out, eps}, N, D, stream, st)) return st;
    GenArgs a{x, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, out, D, eps};
    launch(row_generic<GenKind::LayerNorm>, generic_grid(N), ref_row_threads(D), 0, stream, a, N);
    return launch_status();
}

extern "C" int anima_adaln_layernorm_bf16(const anima_bf16 *x, const anima_bf16 *scale,
                                          const anima_bf16 *shift, anima_bf16 *out, int N, int D,
                                          float eps, anima_stream_t stream) {
    if (int e = check_row_args(N, D)) return e;
    if (N == 0) return ANIMA_OK;
    if (!x || !scale || !shift || !out) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(x) || !bf16_ok(scale) || !bf16_ok(shift) || !bf16_ok(out)) return ANIMA_ERR_MISALIGNED;
    const int64_t n = (int64_t)N * D * 2;
    if (partial_overlap(x, n, out, n)) return ANIMA_ERR_OVERLAP;
    int st;
    if (aligned16(x) && aligned16(out) && aligned16(scale) && aligned16(shift) &&
        dispatch_seg(AdaLNOp<false>{x, scale, shift, out, eps}, N, D, stream, st))
        return st;
    GenArgs a{x, nullptr, nullptr, nullptr, scale, shift, nullptr, out, D, eps};
    launch(row_generic<GenKind::AdaLN>, generic_grid(N), ref_row_threads(D), 0, stream, a, N);
    return launch_status();
}

extern "C" int anima_adaln_layernorm_temb_bf16(const anima_bf16 *x, const anima_bf16 *mod,
                                               const anima_bf16 *temb, anima_bf16 *gate_out, anima_bf16 *out,
                                               int N, int D, float eps, anima_stream_t stream) {
    if (int e = check_row_args(N, D)) return e;
    if (N == 0) return ANIMA_OK;
    if (!x || !mod || !temb || !gate_out || !out) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(x) || !bf16_ok(mod) || !bf16_ok(temb) || !bf16_ok(gate_out) || !bf16_ok(out))
        return ANIMA_ERR_MISALIGNED;
    const int64_t n = (int64_t)N * D * 2, nv = (int64_t)D * 2;
    if (partial_overlap(x, n, out, n)) return ANIMA_ERR_OVERLAP;
    if (overlaps(gate_out, nv, mod, 3 * nv) || overlaps(gate_out, nv, temb, 3 * nv) ||
        overlaps(gate_out, nv, x, n) || overlaps(gate_out, nv, out, n) || overlaps(out, n, mod, 3 * nv) ||
        overlaps(out, n, temb, 3 * nv))
        return ANIMA_ERR_OVERLAP;
    const TembFold fold{temb + D, temb, mod + 2 * D, temb + 2 * D, gate_out};
    int st;
    if (aligned16(x) && aligned16(out) && aligned16(mod) && aligned16(temb) && D % 8 == 0 &&
        dispatch_seg(AdaLNOp<false, true>{x, mod + D, mod, out, eps, fold}, N, D, stream, st))
        return st;
    GenArgs a{x, nullptr, nullptr, nullptr, mod + D, mod, nullptr, out, D, eps, fold};
    launch(row_generic<GenKind::AdaLN>, generic_grid(N), ref_row_threads(D), 0, stream, a, N);
    return launch_status();
}

extern "C" int anima_layer_norm_modulate_bf16(const anima_bf16 *x, const anima_bf16 *scale,
                                              const anima_bf16 *shift, anima_bf16 *out, int N,
                                              int D, float eps, anima_stream_t stream) {
    if (int e = check_row_args(N, D)) return e;
    if (N == 0) return ANIMA_OK;
    if (!x || !scale || !shift || !out) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(x) || !bf16_ok(scale) || !bf16_ok(shift) || !bf16_ok(out)) return ANIMA_ERR_MISALIGNED;
    const int64_t n = (int64_t)N * D * 2;
    if (partial_overlap(x, n, out, n)) return ANIMA_ERR_OVERLAP;
    int st;
    if (aligned16(x) && aligned16(out) && aligned16(scale) && aligned16(shift) &&
        dispatch_seg(AdaLNOp<true>{x, scale, shift, out, eps}, N, D, stream, st))
        return st;
    GenArgs a{x, nullptr, nullptr, nullptr, scale, shift, nullptr, out, D, eps};
    launch(row_generic<GenKind::LnModulate>, generic_grid(N), ref_row_threads(D), 0, stream, a, N);
    return launch_status();
}

extern "C" int anima_residual_gate_adaln_bf16(anima_bf16 *hidden, const anima_bf16 *sub_out,
                                              const anima_bf16 *gate, const anima_bf16 *scale,
                                              const anima_bf16 *shift, anima_bf16 *normed, int N,
                                              int D, float eps, anima_stream_t stream) {
    if (int e = check_row_args(N, D)) return e;
    if (N == 0) return ANIMA_OK;
    if (!hidden || !sub_out || !gate || !scale || !shift || !normed) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(hidden) || !bf16_ok(sub_out) || !bf16_ok(gate) || !bf16_ok(scale) ||
        !bf16_ok(shift) || !bf16_ok(normed))
        return ANIMA_ERR_MISALIGNED;
    const int64_t n = (int64_t)N * D * 2;
    // normed must be a separate buffer from hidden; sub_out may not overlap either output.
    if (partial_overlap(hidden, n, normed, n) || hidden == normed) return ANIMA_ERR_OVERLAP;
    if (partial_overlap(sub_out, n, hidden, n) || partial_overlap(sub_out, n, normed, n))
        return ANIMA_ERR_OVERLAP;
    int st;
    if (aligned16(hidden) && aligned16(sub_out) && aligned16(gate) && aligned16(scale) && aligned16(shift) &&
        aligned16(normed) &&
        dispatch_seg(ResGateAdaLNOp<>{hidden, sub_out, gate, scale, shift, normed, eps}, N, D, stream, st))
        return st;
    GenArgs a{hidden, hidden, sub_out, gate, scale, shift, nullptr, normed, D, eps};
    launch(row_generic<GenKind::ResGate>, generic_grid(N), ref_row_threads(D), 0, stream, a, N);
    return launch_status();
}

extern "C" int anima_residual_gate_adaln_temb_bf16(anima_bf16 *hidden, const anima_bf16 *sub_out,
                                                   const anima_bf16 *gate_in, const anima_bf16 *mod,
                                                   const anima_bf16 *temb, anima_bf16 *gate_out,
                                                   anima_bf16 *normed, int N, int D, float eps,
                                                   anima_stream_t stream) {
    if (int e = check_row_args(N, D)) return e;
    if (N == 0) return ANIMA_OK;
    if (!hidden || !sub_out || !gate_in || !mod || !temb || !gate_out || !normed) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(hidden) || !bf16_ok(sub_out) || !bf16_ok(gate_in) || !bf16_ok(mod) || !bf16_ok(temb) ||
        !bf16_ok(gate_out) || !bf16_ok(normed))
        return ANIMA_ERR_MISALIGNED;
    const int64_t n = (int64_t)N * D * 2, nv = (int64_t)D * 2;
    if (partial_overlap(hidden, n, normed, n) || hidden == normed) return ANIMA_ERR_OVERLAP;
    if (partial_overlap(sub_out, n, hidden, n) || partial_overlap(sub_out, n, normed, n))
        return ANIMA_ERR_OVERLAP;
    // gate_out is written while gate_in, mod and temb are read: it must overlap none of them
    if (overlaps(gate_out, nv, gate_in, nv) || overlaps(gate_out, nv, mod, 3 * nv) ||
        overlaps(gate_out, nv, temb, 3 * nv) || overlaps(gate_out, nv, hidden, n) ||
        overlaps(gate_out, nv, sub_out, n) || overlaps(gate_out, nv, normed, n) ||
        overlaps(hidden, n, mod, 3 * nv) || overlaps(hidden, n, temb, 3 * nv) || overlaps(hidden, n, gate_in, nv) ||
        overlaps(normed, n, mod, 3 * nv) || overlaps(normed, n, temb, 3 * nv) || overlaps(normed, n, gate_in, nv))
        return ANIMA_ERR_OVERLAP;
    const TembFold fold{temb + D, temb, mod + 2 * D, temb + 2 * D, gate_out};
    int st;
    if (aligned16(hidden) && aligned16(sub_out) && aligned16(gate_in) && aligned16(mod) && aligned16(temb) &&
        aligned16(normed) && D % 8 == 0 &&
        dispatch_seg(ResGateAdaLNOp<true>{hidden, sub_out, gate_in, mod + D, mod, normed, eps, fold}, N, D, stream, st))
        return st;
    GenArgs a{hidden, hidden, sub_out, gate_in, mod + D, mod, nullptr, normed, D, eps, fold};
    launch(row_generic<GenKind::ResGate>, generic_grid(N), ref_row_threads(D), 0, stream, a, N);
    return launch_status();
}

extern "C" int anima_rms_norm_bf16(const anima_bf16 *x, const anima_bf16 *weight, anima_bf16 *out,
                                   int N, int D, float eps, anima_stream_t stream) {
    if (int e = check_row_args(N, D)) return e;
    if (N == 0) return ANIMA_OK;
    if (!x || !out) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(x) || !bf16_ok(out) || (weight && !bf16_ok(weight))) return ANIMA_ERR_MISALIGNED;
    const int64_t n = (int64_t)N * D * 2;
    if (partial_overlap(x, n, out, n)) return ANIMA_ERR_OVERLAP;
    int st;
    if (aligned16(x) && aligned16(out) && (!weight || aligned16(weight)) && (D == 64 || D == 128 || D == 256)) {
        const unsigned grid = (unsigned)((N + kRowBlock / 8 - 1) / (kRowBlock / 8));
        switch (D) {
#define ANIMA_RMS_SMALL(Dv, Kv)                                                                          \
    case Dv:                                                                                            \
        if (weight) launch(rms_small<Kv, true>, grid, kRowBlock, 0, stream, x, weight, out, (int64_t)N, D, eps);  \
        else launch(rms_small<Kv, false>, grid, kRowBlock, 0, stream, x, weight, out, (int64_t)N, D, eps);        \
        break;
            ANIMA_RMS_SMALL(64, 1) ANIMA_RMS_SMALL(128, 2) ANIMA_RMS_SMALL(256, 4)
#undef ANIMA_RMS_SMALL
        }
        return launch_status();
    }
    if (aligned16(x) && aligned16(out) && (!weight || aligned16(weight))) {
        const bool done = weight ? dispatch_seg(RmsOp<true>{x, weight, out, eps}, N, D, stream, st)
                                 : dispatch_seg(RmsOp<false>{x, weight, out, eps}, N, D, stream, st);
        if (done) return st;
    }
    GenArgs a{x, nullptr, nullptr, nullptr, nullptr, nullptr, weight, out, D, eps};
    launch(row_generic<GenKind::Rms>, generic_grid(N), ref_row_threads(D), 0, stream, a, N);
    return launch_status();
}

extern "C" int anima_adaln_rms_norm_bf16(const anima_bf16 *x, const anima_bf16 *scale,
                                         const anima_bf16 *shift, anima_bf16 *out, int N, int D,
                                         float eps, anima_stream_t stream) {
    if (int e = check_row_args(N, D)) return e;
    if (N == 0) return ANIMA_OK;
    if (!x || !scale || !shift || !out) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(x) || !bf16_ok(scale) || !bf16_ok(shift) || !bf16_ok(out)) return ANIMA_ERR_MISALIGNED;
    const int64_t n = (int64_t)N * D * 2;
    if (partial_overlap(x, n, out, n) || partial_overlap(scale, n, out, n) ||
        partial_overlap(shift, n, out, n))
        return ANIMA_ERR_OVERLAP;
    int st;
    if (aligned16(x) && aligned16(out) && aligned16(scale) && aligned16(shift) &&
        dispatch_seg(AdaRmsOp{x, scale, shift, out, eps}, N, D, stream, st))
        return st;
    GenArgs a{x, nullptr, nullptr, nullptr, scale, shift, nullptr, out, D, eps};
    launch(row_generic<GenKind::AdaRms>, generic_grid(N), ref_row_threads(D), 0, stream, a, N);
    return launch_status();
}

extern "C" int anima_gemma_rms_norm_bf16(const anima_bf16 *x, const anima_bf16 *weight,
                                         anima_bf16 *out, int N, int D, float eps,
                                         anima_stream_t stream) {
    if (N < 0 || D <= 0) return ANIMA_ERR_BAD_SHAPE;
    if (N == 0) return ANIMA_OK;
    if (!x || !weight || !out) return ANIMA_ERR_NULL_POINTER;
    if (!bf16_ok(x) || !bf16_ok(weight) || !bf16_ok(out)) return ANIMA_ERR_MISALIGNED;
    const int64_t n = (int64_t)N * D * 2;
    if (partial_overlap(x, n, out, n)) return ANIMA_ERR_OVERLAP;
    int threads = (D <= 1024) ? ((D + 31) / 32 * 32) : 1024;
    launch(gemma_rms_generic, generic_grid(N), threads, 0, stream, x, weight, out, (int64_t)N, D, eps);
    return launch_status();
}
