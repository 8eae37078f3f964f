// tcgen05 building blocks shared by the prefill GEMM, the batched decode projections and the local
// stacks' projections: bounded mbarrier waits, 2-D TMA loads (no multicast), shared-memory and
// instruction descriptors for kind::f16 with bf16 or f16 operands, the MMA, its commit, TMEM loads,
// and the host's tensor maps.
#pragma once

#include <cuda.h>

#include <mutex>

#include "tg_common.cuh"
#include "tg_internal.h"

namespace tg {

// Waits for the phase of parity `parity` of `bar` to complete, for at most 2 s (1 ms once the
// block has given up on a wait). Past that it records ERR_WAIT_TIMEOUT and returns, so that the
// kernel always ends.
TG_DEVICE void mbar_wait(uint32_t bar, uint32_t parity, uint32_t *err, volatile int *gave_up) {
    if (mbar_try_wait(bar, parity)) return;
    const uint64_t limit = *gave_up ? 1000000ull : 2000000000ull;
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer() - t0 > limit) {
            *gave_up = 1;
            atomicExch(err, ERR_WAIT_TIMEOUT);
            return;
        }
    }
}

TG_DEVICE void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

TG_DEVICE void tma_load_3d(uint32_t dst, const CUtensorMap *map, int x, int y, int z, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
        : "memory");
}

// The shared-memory matrix descriptor of a K-major tile with 128-byte rows in the 128-byte
// swizzle TMA writes: start address, leading byte offset 16 (unused for this layout), stride
// byte offset 1024 between groups of 8 rows, descriptor version 1, swizzle mode 2 (128 B).
TG_DEVICE uint64_t sw128_desc(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3fff) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// The instruction descriptor of kind::f16 with bf16 A and B (both K-major), f32 D, M x N.
__host__ __device__ constexpr uint32_t bf16_idesc(int m, int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// The instruction descriptor of kind::f16 with f16 A and B (both K-major), f32 D, M x N.
__host__ __device__ constexpr uint32_t f16_idesc(int m, int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

TG_DEVICE void tc_mma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

// The same MMA with A read from TMEM (tmem_a: lane 0 and the first column; row i of A in lane i,
// its K values two to a 32-bit column, the lower-indexed in the low half): no shared-memory read
// for A.
TG_DEVICE void tc_mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

TG_DEVICE void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// ---- pairs of CTAs (a cluster of two on one TPC, tcgen05 cta_group::2) ----------------------------
// The MMA issued by the pair's leader (rank 0) reads A's 128 rows and half of B's N from each CTA's
// shared memory at the same offsets and writes each CTA's 128 rows of D into its own TMEM.

TG_DEVICE uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// Every thread of both CTAs: the pair's barriers, shared memory and TMEM are past this point in both.
TG_DEVICE void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
TG_DEVICE void tc_mma2(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}
// The leader's MMAs so far done: one arrival on the barrier at `bar`'s offset in each CTA of the
// pair (a commit to each: the leader's own, and the peer's through its cluster address).
TG_DEVICE void tc_commit2(uint32_t bar) {
    uint32_t peer;
    asm volatile("mapa.shared::cluster.u32 %0, %1, 1;" : "=r"(peer) : "r"(bar));
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(peer) : "memory");
}
// A 2-D TMA load into this CTA's shared memory whose bytes complete on the leader CTA's barrier at
// `bar`'s offset (no multicast).
TG_DEVICE void tma_load_2d_pair(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar & 0xFEFFFFFFu)
        : "memory");
}
// One arrival on the barrier at `bar`'s offset in CTA `rank` of the cluster.
TG_DEVICE void mbar_arrive_remote(uint32_t bar, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(bar), "r"(rank));
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(r) : "memory");
}

TG_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
TG_DEVICE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// Issues a load of 16 consecutive f32 columns of this warp's 32 TMEM lanes without waiting for it
// (tmem_wait_ld before the registers are read): several loads then share one wait.
TG_DEVICE void tmem_ld16_nowait(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
TG_DEVICE void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 16 TMEM lanes x 32 columns (taddr's lane and up): lane t of the warp gets, of column group k
// (columns 8 k .. 8 k + 7), r[4 k], r[4 k + 1] = row t / 4, columns 8 k + 2 (t % 4) and the next,
// and r[4 k + 2], r[4 k + 3] = row t / 4 + 8, the same columns (mma.sync's accumulator layout).
TG_DEVICE void tmem_ld16x256_nowait(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile("tcgen05.ld.sync.aligned.16x256b.x4.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
                   "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr));
}

// Stores 16 consecutive f32 columns of this warp's 32 TMEM lanes (lane i of the warp to row
// (warp % 4) * 32 + i); tmem_wait_st before anything else reads or writes them.
TG_DEVICE void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
TG_DEVICE void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 16 consecutive f32 columns of this warp's 32 TMEM lanes: lane i of the warp gets row
// (warp % 4) * 32 + i.
TG_DEVICE void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// ---- host ---------------------------------------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void *p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// A 2-D map over a row-major [rows][k] matrix of 2-byte elements (bf16 or f16), boxes of 64 columns
// x `box_rows` rows in the 128-byte swizzle; rows past `rows` read as zero.
inline bool make_map_2byte(CUtensorMap *map, const void *ptr, uint64_t rows, uint64_t k, uint32_t box_rows,
                           CUtensorMapDataType type) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {k, rows};
    cuuint64_t strides[1] = {k * 2};
    cuuint32_t box[2] = {64, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, type, 2, const_cast<void *>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

inline bool make_map_bf16(CUtensorMap *map, const void *ptr, uint64_t rows, uint64_t k, uint32_t box_rows) {
    return make_map_2byte(map, ptr, rows, k, box_rows, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);
}

inline bool make_map_f16(CUtensorMap *map, const void *ptr, uint64_t rows, uint64_t k, uint32_t box_rows) {
    return make_map_2byte(map, ptr, rows, k, box_rows, CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
}

// A 3-D map over an f16 matrix of `rows` rows and k columns stored k-block-major, [k / 64][rows]
// [64]: boxes of 64 columns x `box_rows` rows x `box_kb` k-blocks, in the 128-byte swizzle (each
// k-block's rows one after another, as a 2-D box of the same rows lays them out); rows past `rows`
// read as zero.
inline bool make_map_f16_blocked(CUtensorMap *map, const void *ptr, uint64_t rows, uint64_t k, uint32_t box_rows,
                                 uint32_t box_kb) {
    EncodeTiledFn fn = encode_fn();
    if (!fn || k % 64) return false;
    cuuint64_t dims[3] = {64, rows, k / 64};
    cuuint64_t strides[2] = {128, rows * 128};
    cuuint32_t box[3] = {64, box_rows, box_kb};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(ptr), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace tg
