// gather.cu -- token-embedding gather (sm_100a), bit-exact.
//
// One warp per token: the id is read once (a broadcast load), then the row is copied in
// 16-byte chunks, four per lane issued back to back before any store, so a 2 KB Qwen3
// row (D = 1024) moves with one round trip. Ids outside [0, vocab) yield a zero row and
// are counted instead of reading out of bounds; the reference does no check
// (gemma_ops.cu:34-45).
#include "common.cuh"

namespace anima {
namespace {

constexpr int kGatherBlock = 256;
constexpr int kGatherU = 4;

struct GatherArgs {
    const anima_bf16 *table;
    const int32_t *ids;
    anima_bf16 *out;
    int T, D, vocab;
    int32_t *bad;
};

__global__ void __launch_bounds__(kGatherBlock) gather_vec(GatherArgs a) {
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int64_t t = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (t >= a.T) return;
    const int id = __ldg(a.ids + t);
    const bool ok = a.vocab <= 0 || (id >= 0 && id < a.vocab);
    if (!ok && lane == 0 && a.bad) atomicAdd(a.bad, 1);
    const int nch = a.D / 8;
    const anima_bf16 *src = a.table + (int64_t)id * a.D;
    anima_bf16 *dst = a.out + t * a.D;
    for (int c0 = lane; c0 < nch; c0 += 32 * kGatherU) {
        Vec8 v[kGatherU];
#pragma unroll
        for (int u = 0; u < kGatherU; ++u) {
            const int c = c0 + 32 * u;
            v[u] = Vec8{{0u, 0u, 0u, 0u}};
            if (ok && c < nch) v[u] = ld_stream(src + (int64_t)c * 8);
        }
#pragma unroll
        for (int u = 0; u < kGatherU; ++u) {
            const int c = c0 + 32 * u;
            if (c < nch) st_vec(dst + (int64_t)c * 8, v[u]);
        }
    }
}

// Any D and 2-byte alignment: element copies.
__global__ void gather_scalar(GatherArgs a) {
    pdl_wait();
    const int64_t t = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (t >= a.T) return;
    const int lane = threadIdx.x & 31;
    const int id = a.ids[t];
    const bool ok = a.vocab <= 0 || (id >= 0 && id < a.vocab);
    if (!ok && lane == 0 && a.bad) atomicAdd(a.bad, 1);
    for (int d = lane; d < a.D; d += 32) a.out[t * a.D + d] = ok ? a.table[(int64_t)id * a.D + d] : (anima_bf16)0;
}

}  // namespace
}  // namespace anima

using namespace anima;

extern "C" int anima_embedding_lookup_bf16(const anima_bf16 *table, const int32_t *ids, anima_bf16 *out,
                                           int T, int D, int vocab, int32_t *bad_id_count,
                                           anima_stream_t stream) {
    if (T < 0 || D <= 0) return ANIMA_ERR_BAD_SHAPE;
    if (T == 0) return ANIMA_OK;
    if (!table || !ids || !out) return ANIMA_ERR_NULL_POINTER;
    if (!aligned_to(table, 2) || !aligned_to(out, 2) || !aligned_to(ids, 4) ||
        (bad_id_count && !aligned_to(bad_id_count, 4)))
        return ANIMA_ERR_MISALIGNED;
    if (partial_overlap(out, (int64_t)T * D * 2, ids, (int64_t)T * 4) || (const void *)out == ids)
        return ANIMA_ERR_OVERLAP;
    // Rows written while other warps still read the table would race.
    if (vocab > 0 && overlaps(out, (int64_t)T * D * 2, table, (int64_t)vocab * D * 2)) return ANIMA_ERR_OVERLAP;
    GatherArgs a{table, ids, out, T, D, vocab, bad_id_count};
    const int64_t per_block = kGatherBlock / 32;
    const unsigned grid = (unsigned)((T + per_block - 1) / per_block);
    if (D % 8 == 0 && aligned16(table) && aligned16(out))
        launch(gather_vec, grid, kGatherBlock, 0, stream, a);
    else
        launch(gather_scalar, grid, kGatherBlock, 0, stream, a);
    return launch_status();
}
