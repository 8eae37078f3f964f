// The prefill's projection GEMM, C[m][n] = A[m][k] B[n][k]^T with f32 accumulation
// (kernels/gpu/gemm.mlir:14-29; a linear layer: A the activations, B the weights as a checkpoint
// lays them out, both K-major).
//
// bf16: a tcgen05 kernel. Each block computes a 128 x BN tile of C. One thread streams A and B
// tiles of 64 columns of K into a ring of shared-memory stages with TMA (128-byte swizzle, no
// multicast), one thread issues tcgen05.mma into a TMEM accumulator (M = 128, N = BN, K = 16 per
// instruction) and releases each stage with tcgen05.commit, and all four warps read the
// accumulator back with tcgen05.ld for the epilogue. Every wait on an mbarrier is bounded: past
// its limit the kernel sets the context's error word and runs to its end.
//
// f32: a SIMT kernel, each sum sequential in k.
#include "tc_common.cuh"

namespace tg {

// ---- f32 SIMT ---------------------------------------------------------------------------------

__global__ void __launch_bounds__(256)
    gemm_f32_kernel(int M, int N, int K, const float *__restrict__ A, const float *__restrict__ B,
                    float *__restrict__ C) {
    __shared__ float As[16][64 + 4];
    __shared__ float Bs[16][64 + 4];
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += 16) {
        for (int i = threadIdx.x; i < 64 * 16; i += 256) {
            const int r = i / 16, kk = i % 16;
            As[kk][r] = (m0 + r < M && k0 + kk < K) ? A[(size_t)(m0 + r) * K + k0 + kk] : 0.0f;
            Bs[kk][r] = (n0 + r < N && k0 + kk < K) ? B[(size_t)(n0 + r) * K + k0 + kk] : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; kk++) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                a[i] = As[kk][ty * 4 + i];
                b[i] = Bs[kk][tx * 4 + i];
            }
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int m = m0 + ty * 4 + i;
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int n = n0 + tx * 4 + j;
            if (n < N) C[(size_t)m * N + n] = acc[i][j];
        }
    }
}

// ---- tcgen05 bf16 ------------------------------------------------------------------------------

constexpr int TC_BM = 128, TC_BK = 64;
constexpr int TC_A_BYTES = TC_BM * TC_BK * 2;  // 16 KiB per stage


// A stage: the tile's A (128 rows) and B (BN rows, or with CG = 2 this CTA's half of them).
template <int BN, int CG = 1>
struct TcLayout {
    static constexpr int B_BYTES = BN / CG * TC_BK * 2;
    static constexpr int STAGE = TC_A_BYTES + B_BYTES;
    static constexpr int STAGES = (4 * (TC_A_BYTES + 256 * TC_BK * 2)) / STAGE;  // 192 KiB of stages
    static constexpr int BARRIERS = STAGES * STAGE;                           // offset of the mbarriers
    static constexpr int SMEM = BARRIERS + 256 + 1024;                        // + alignment slack
    // (with the 1 KiB of static shared memory the kernel also takes)
    static_assert(SMEM + 1024 <= 227 * 1024, "the stages and barriers fit a block's shared memory");
};

// Epilogues: C in f32, or (B's rows in gate_up_row's order: blocks of 128 gate rows, then the same
// outputs' 128 up rows) SiLU(gate) up in bf16, a tile's B loaded as two boxes of BN / 2 rows — the
// gate rows of BN / 2 outputs, then their up rows — so that columns c and BN / 2 + c of the
// accumulator are one output's gate and up, or (B the
// q/k/v projection) rope_rows.comp's work: RoPE on each head's column pairs (i, i + hd/2), q rows
// stored bf16, k and v rows appended to the cache at the row's position and slot.
// TC_EPI_RES: C = residual + s C in f32, add_norm_rows.comp's sum (the same fused multiply-add),
// stored in place of C.
enum { TC_EPI_F32 = 0, TC_EPI_SILU = 1, TC_EPI_ROPE = 2, TC_EPI_RES = 3 };

// 32 bytes of a lane's row at dst (global memory): one 256-bit store, a whole sector, where dst is
// 32-byte aligned, else two 16-byte stores (a binding need only be 16-byte aligned). A warp of such
// stores, a row a lane, then asks L2 for 32 whole sectors rather than 64 halves.
TG_DEVICE void st_row32(void *dst, uint4 a, uint4 b) {
    if ((reinterpret_cast<uintptr_t>(dst) & 31) == 0) {
        asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(dst), "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w),
                     "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w)
                     : "memory");
    } else {
        reinterpret_cast<uint4 *>(dst)[0] = a;
        reinterpret_cast<uint4 *>(dst)[1] = b;
    }
}

struct EpiArgs {
    tg_params p;
    const uint32_t *at;
    const float *cosv, *sinv;
    bf16 *q, *kc, *vc;
    const float *res;  // TC_EPI_RES: [M][N] f32, scaled by p.residual_scale
};

// Persistent: one block per SM walks tiles t = blockIdx.x, + gridDim.x, ... within a part of K,
// over the smaller operand fastest: the tiles at work at one time then share the few row panels
// of the larger operand, which streams from HBM once, and re-read the smaller from L2 (n fastest
// when N <= M, as every prefill projection's weights against its 32,768 rows: m fastest read
// down's 268 MB of A four times from HBM, once for each 256-wide column of tiles). With `parts` > 1 (f32 epilogue
// only) K is cut into that many equal ranges and tile (m, n, part) stores its partial sum at
// C[part][m][n]; the kernel that reads C adds the parts in part order, so a row's sums depend on
// the shape and the part count, never on how many rows a launch takes. Warp 0 streams A and B tiles into a ring of stages with
// TMA; warp 1 owns TMEM (two accumulators of BN columns) and issues the MMAs; warps 2-5 drain an
// accumulator (tcgen05.ld) and store it while the MMAs fill the other, so that a tile's epilogue
// overlaps the next tile's main loop.
// Epilogue warps: four (one to each quadrant of TMEM lanes) for a single CTA - the batched
// decoder's narrow, latency-bound tiles - and eight for a pair (two to each quadrant, one to each
// half of the tile's columns: a short main loop, as the prefill gate/up's K = 1024, would
// otherwise wait on SiLU's epilogue).
template <int CG>
constexpr int tc_epi_warps() { return 4 * CG; }
template <int CG>
constexpr int tc_threads() { return (2 + tc_epi_warps<CG>()) * 32; }

//
// CG = 2: the grid is pairs of CTAs (clusters of two), a pair taking tiles of 256 rows: each CTA
// loads its 128 rows of A and half of B's BN rows (for SiLU, CTA 0 the gate rows and CTA 1 the up
// rows of the tile's outputs), all the copies completing on the leader's (rank 0) barrier, which
// expects both CTAs' bytes; the leader's MMA thread issues tcgen05.mma.cta_group::2 (M = 256) and
// commits to the barriers of both CTAs; each CTA's epilogue drains its own TMEM rows as with
// CG = 1 and releases the accumulator on the leader's barrier. Per stage an SM then reads
// 128 + BN / 2 rows of K for 128 x BN outputs instead of 128 + BN.
template <int BN, int EPI = TC_EPI_F32, int CG = 1>
__global__ void __launch_bounds__(tc_threads<CG>(), 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                   void *__restrict__ Cout, int M, int N, int K, uint32_t *err, const __grid_constant__ EpiArgs re,
                   int b_const, int parts) {
    static_assert(CG == 1 || CG == 2, "one CTA or a pair");
    using L = TcLayout<BN, CG>;
    constexpr int S = L::STAGES;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t base = smem_u32(smem);
    const uint32_t bars = base + L::BARRIERS;
    auto full = [&](int s) { return bars + 8u * s; };
    auto empty = [&](int s) { return bars + 8u * (S + s); };
    auto acc_full = [&](int a) { return bars + 8u * (2 * S + a); };
    auto acc_empty = [&](int a) { return bars + 8u * (2 * S + 2 + a); };
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::BARRIERS + 8 * (2 * S + 4));
    __shared__ int gave_up;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = CG == 2 ? cluster_rank() : 0u;
    const int cta = CG == 2 ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;  // the pair's (or the CTA's) index
    const int ctas = CG == 2 ? (int)(gridDim.x >> 1) : (int)gridDim.x;
    constexpr int TM = TC_BM * CG;  // rows a tile
    const int mt = (M + TM - 1) / TM, nt = N / BN, per = mt * nt, tiles = per * parts;
    const int nk = K / TC_BK / parts;  // k-blocks a tile
    const bool n_fast = N <= M;
    auto m_of = [&](int t) { return n_fast ? (t % per) / nt : t % mt; };
    auto m0_of = [&](int t) { return m_of(t) * TM + (int)rank * TC_BM; };  // this CTA's first row
    auto n0_of = [&](int t) { return (n_fast ? (t % per) % nt : (t % per) / mt) * BN; };
    auto kb0_of = [&](int t) { return (t / per) * nk; };  // the tile's first k-block
    auto load_a = [&](uint32_t dst, int kx, int m0, uint32_t bar) {
        if constexpr (CG == 2)
            tma_load_2d_pair(dst, &map_a, kx, m0, bar);
        else
            tma_load_2d(dst, &map_a, kx, m0, bar);
    };
    // A stage's B tile: BN rows from n0, or (SiLU) the gate rows of outputs n0 / 2 .. + BN / 2 and
    // then their up rows; with CG = 2 this CTA's half of them.
    auto load_b = [&](uint32_t dst, int kx, int n0, uint32_t bar) {
        if constexpr (CG == 2) {
            int row = n0 + (int)rank * (BN / 2);
            if constexpr (EPI == TC_EPI_SILU) {
                static_assert(BN == 256, "a pair's SiLU tile: 128 gate rows in one CTA, their 128 up rows in the other");
                row = (n0 / 2 / 128) * 256 + (int)rank * 128;
            }
            tma_load_2d_pair(dst, &map_b, kx, row, bar);
        } else if constexpr (EPI == TC_EPI_SILU) {
            const int o0 = n0 / 2, gate = (o0 / 128) * 256 + o0 % 128;
            tma_load_2d(dst, &map_b, kx, gate, bar);
            tma_load_2d(dst + (BN / 2) * TC_BK * 2, &map_b, kx, gate + 128, bar);
        } else {
            tma_load_2d(dst, &map_b, kx, n0, bar);
        }
    };
    pdl_launch_dependents();

    if (threadIdx.x == 0) {
        gave_up = 0;
        for (int s = 0; s < S; s++) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(acc_full(a), 1);
            // CG = 1: every epilogue thread; CG = 2: one thread of each CTA's epilogue, on the leader's.
            mbar_init(acc_empty(a), CG == 2 ? 2 : tc_epi_warps<CG>() * 32);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_b)) : "memory");
    }
    if (warp == 1) {
        if constexpr (CG == 2) {  // warp 1 of both CTAs
            asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                         "r"((uint32_t)(2 * BN))
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
        } else {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                         "r"((uint32_t)(2 * BN))
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        }
    }
    tc_fence_before();
    if constexpr (CG == 2)
        cluster_sync();  // both CTAs' barriers are initialised before either's copies or commits reach them
    else
        __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // Producer: k-block g (over all this block's tiles) into stage g % S once its MMAs
            // have released it. When B is a weight (constant for the program), the first tile's
            // first stages of B are loaded before the wait on the kernel before it, so that they
            // stream while that kernel finishes; A, that kernel's output, after the wait.
            // With CG = 2 only the leader expects (both CTAs' bytes, on its barrier).
            auto expect = [&](int s) {
                if (rank == 0) mbar_arrive_expect_tx(full(s), CG * L::STAGE);
            };
            const int pre = b_const && cta < tiles ? (nk < S ? nk : S) : 0;
            for (int kb = 0; kb < pre; kb++) {
                expect(kb);
                load_b(base + kb * L::STAGE + TC_A_BYTES, (kb0_of(cta) + kb) * TC_BK, n0_of(cta), full(kb));
            }
            pdl_wait();
            int g = 0;
            for (int t = cta; t < tiles; t += ctas) {
                const int m0 = m0_of(t), n0 = n0_of(t), kb0 = kb0_of(t);
                for (int kb = 0; kb < nk; kb++, g++) {
                    const int s = g % S, kx = (kb0 + kb) * TC_BK;
                    if (g < pre) {  // B is in flight already
                        load_a(base + s * L::STAGE, kx, m0, full(s));
                        continue;
                    }
                    mbar_wait(empty(s), ((g / S) & 1) ^ 1, err, &gave_up);
                    expect(s);
                    load_a(base + s * L::STAGE, kx, m0, full(s));
                    load_b(base + s * L::STAGE + TC_A_BYTES, kx, n0, full(s));
                }
            }
            // Every copy this thread started has landed before the block can end: on the leader's
            // full barriers, or (the other CTA of a pair) once the MMAs that read them released
            // this CTA's stages.
            for (int h = g > S ? g - S : 0; h < g; h++) {
                if (rank == 0)
                    mbar_wait(full(h % S), (h / S) & 1, err, &gave_up);
                else
                    mbar_wait(empty(h % S), (h / S) & 1, err, &gave_up);
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            // MMA issuer (the leader of a pair): tile i into accumulator i % 2 once the epilogue
            // (both CTAs' with CG = 2) has drained it.
            constexpr uint32_t idesc = bf16_idesc(TM, BN);
            int g = 0, i = 0;
            for (int t = cta; t < tiles; t += ctas, i++) {
                const int acc = i & 1;
                mbar_wait(acc_empty(acc), ((i >> 1) & 1) ^ 1, err, &gave_up);
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(acc * BN);
                for (int kb = 0; kb < nk; kb++, g++) {
                    const int s = g % S;
                    mbar_wait(full(s), (g / S) & 1, err, &gave_up);
                    tc_fence_after();
                    const uint32_t a_addr = base + s * L::STAGE;
                    const uint32_t b_addr = a_addr + TC_A_BYTES;
#pragma unroll
                    for (int k = 0; k < TC_BK / 16; k++) {
                        if constexpr (CG == 2)
                            tc_mma2(d, sw128_desc(a_addr + k * 32), sw128_desc(b_addr + k * 32), idesc,
                                    (kb > 0 || k > 0) ? 1u : 0u);
                        else
                            tc_mma(d, sw128_desc(a_addr + k * 32), sw128_desc(b_addr + k * 32), idesc,
                                   (kb > 0 || k > 0) ? 1u : 0u);
                    }
                    if constexpr (CG == 2)
                        tc_commit2(empty(s));
                    else
                        tc_commit(empty(s));
                }
                if constexpr (CG == 2)
                    tc_commit2(acc_full(acc));
                else
                    tc_commit(acc_full(acc));
            }
        }
    } else {
        // Epilogue: warp w drains TMEM lanes (w % 4) * 32 .. + 31, i.e. rows m0 + that of the tile,
        // columns of half eh of the tile (for RoPE: half of its heads, or of a head's pair columns).
        constexpr int EH = tc_epi_warps<CG>() / 4;  // column parts: each a warp per TMEM lane quadrant
        const int q = warp & 3, eh = (warp - 2) / 4;
        const uint32_t lane_off = (uint32_t)(q * 32) << 16;
        int i = 0;
        for (int t = cta; t < tiles; t += ctas, i++) {
            const int acc = i & 1;
            const int m0 = m0_of(t), n0 = n0_of(t);
            mbar_wait(acc_full(acc), (i >> 1) & 1, err, &gave_up);
            tc_fence_after();
            const int row = m0 + q * 32 + lane;
            const uint32_t lane_base = tmem + lane_off + (uint32_t)(acc * BN);
            if constexpr (EPI == TC_EPI_ROPE) {
                static_assert(BN % 64 == 0, "whole heads a tile");
                const tg_params &p = re.p;
                const int hd = p.head_dim, half = hd / 2, heads = p.heads, kvh = p.kv_heads;
                uint32_t pos = 0, slot = 0;
                const bool ok = row < M && placed(re.at, p.rows, row, p.capacity, p.slots, pos, slot);
                // 16 pair columns at a time: the row's cos and sin for them once (every head of the
                // tile shares the position), then each head's pairs.
                const bool by_heads = BN / hd >= 2;  // else one head: the halves split its pair columns
                const int c_lo = by_heads ? 0 : eh * (half / EH), c_hi = by_heads ? half : c_lo + half / EH;
                const int h_lo = by_heads ? eh * (BN / EH) : 0, h_hi = by_heads ? h_lo + BN / EH : BN;
#pragma unroll 1
                for (int c0 = c_lo; c0 < c_hi; c0 += 16) {
                    float cs[16], sn[16];
                    if (ok && p.rope) {
                        const float4 *c4 = reinterpret_cast<const float4 *>(re.cosv + (size_t)pos * half + c0);
                        const float4 *s4 = reinterpret_cast<const float4 *>(re.sinv + (size_t)pos * half + c0);
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            const float4 cv = __ldg(c4 + e), sv = __ldg(s4 + e);
                            cs[4 * e] = cv.x, cs[4 * e + 1] = cv.y, cs[4 * e + 2] = cv.z, cs[4 * e + 3] = cv.w;
                            sn[4 * e] = sv.x, sn[4 * e + 1] = sv.y, sn[4 * e + 2] = sv.z, sn[4 * e + 3] = sv.w;
                        }
                    }
#pragma unroll 1
                    for (int hb = h_lo; hb < h_hi; hb += hd) {
                        const int head = (n0 + hb) / hd;
                        uint32_t va[16], vb[16];
                        tmem_ld16_nowait(lane_base + hb + c0, va);
                        tmem_ld16_nowait(lane_base + hb + half + c0, vb);
                        tmem_wait_ld();
                        if (!ok) continue;
                        float a[16], b[16];
#pragma unroll
                        for (int e = 0; e < 16; e++) {
                            a[e] = __uint_as_float(va[e]);
                            b[e] = __uint_as_float(vb[e]);
                        }
                        if (head < heads + kvh && p.rope) {
                            // As upstream: x cos + rotate_half(x) sin (rope_rows.comp:33-70).
#pragma unroll
                            for (int e = 0; e < 16; e++) {
                                const float na = __fmaf_rn(a[e], cs[e], -__fmul_rn(b[e], sn[e]));
                                const float nb = __fmaf_rn(b[e], cs[e], __fmul_rn(a[e], sn[e]));
                                a[e] = na;
                                b[e] = nb;
                            }
                        }
                        bf16 *dst;
                        if (head < heads)
                            dst = re.q + ((size_t)row * heads + head) * hd;
                        else if (head < heads + kvh)
                            dst = re.kc + (((size_t)slot * kvh + (head - heads)) * p.capacity + pos) * hd;
                        else
                            dst = re.vc + (((size_t)slot * kvh + (head - heads - kvh)) * p.capacity + pos) * hd;
                        uint32_t wa[8], wb[8];
#pragma unroll
                        for (int e = 0; e < 8; e++) {
                            const __nv_bfloat162 x = __floats2bfloat162_rn(a[2 * e], a[2 * e + 1]);
                            const __nv_bfloat162 y = __floats2bfloat162_rn(b[2 * e], b[2 * e + 1]);
                            wa[e] = *reinterpret_cast<const uint32_t *>(&x);
                            wb[e] = *reinterpret_cast<const uint32_t *>(&y);
                        }
                        st_row32(dst + c0, make_uint4(wa[0], wa[1], wa[2], wa[3]), make_uint4(wa[4], wa[5], wa[6], wa[7]));
                        st_row32(dst + half + c0, make_uint4(wb[0], wb[1], wb[2], wb[3]), make_uint4(wb[4], wb[5], wb[6], wb[7]));
                    }
                }
            } else if constexpr (EPI == TC_EPI_SILU) {
                static_assert(BN % 32 == 0 && 128 % (BN / 2) == 0, "gate and up halves of whole 16-column loads");
                bf16 *out = static_cast<bf16 *>(Cout);
                const int inner = N / 2;
#pragma unroll 1
                for (int c0 = eh * (BN / 2 / EH); c0 < (eh + 1) * (BN / 2 / EH); c0 += 16) {
                    uint32_t g[16], u[16];
                    tmem_ld16_nowait(lane_base + c0, g);
                    tmem_ld16_nowait(lane_base + BN / 2 + c0, u);
                    tmem_wait_ld();
                    if (row < M) {
                        uint32_t packed[8];
#pragma unroll
                        for (int e = 0; e < 8; e++) {
                            const __nv_bfloat162 v = __floats2bfloat162_rn(
                                silu_mul(__uint_as_float(g[2 * e]), __uint_as_float(u[2 * e])),
                                silu_mul(__uint_as_float(g[2 * e + 1]), __uint_as_float(u[2 * e + 1])));
                            packed[e] = *reinterpret_cast<const uint32_t *>(&v);
                        }
                        st_row32(out + (size_t)row * inner + n0 / 2 + c0, make_uint4(packed[0], packed[1], packed[2], packed[3]),
                                 make_uint4(packed[4], packed[5], packed[6], packed[7]));
                    }
                }
            } else {
                // The warp's 32 rows in two 16-row halves by TMEM's 16x256b shape (a row's 8 columns
                // of a group over 4 lanes): each 8-byte store - and residual load - of the warp covers
                // 8 rows' 32 consecutive bytes, whole sectors, where a row a lane's float4 touched 32
                // rows' half sectors (config 4's prefill: o 3.1 -> 2.2 ms; down 4.9 -> 4.8 ms against
                // a transpose through shared memory, which o's short main loop could not hide).
                float *C = static_cast<float *>(Cout) + (size_t)(t / per) * M * N;
                const float sc = re.p.residual_scale;
                const int rt = lane >> 2, ct = 2 * (lane & 3), rbase = m0 + q * 32;
#pragma unroll 1
                for (int c0 = eh * (BN / EH); c0 < (eh + 1) * (BN / EH); c0 += 32) {
                    float2 r[2][2][4];  // [half][row of the lane's two][column group]
                    if constexpr (EPI == TC_EPI_RES) {  // the residual's columns, loaded under the TMEM loads
#pragma unroll
                        for (int hh = 0; hh < 2; hh++)
#pragma unroll
                            for (int s = 0; s < 2; s++) {
                                const int rr = rbase + 16 * hh + 8 * s + rt;
#pragma unroll
                                for (int k = 0; k < 4; k++)
                                    r[hh][s][k] = rr < M ? __ldg(reinterpret_cast<const float2 *>(re.res + (size_t)rr * N + n0 + c0 +
                                                                                                  8 * k + ct))
                                                         : make_float2(0.f, 0.f);
                            }
                    }
                    uint32_t v[2][16];
                    tmem_ld16x256_nowait(lane_base + c0, v[0]);
                    tmem_ld16x256_nowait(lane_base + (16u << 16) + c0, v[1]);
                    tmem_wait_ld();
#pragma unroll
                    for (int hh = 0; hh < 2; hh++)
#pragma unroll
                        for (int s = 0; s < 2; s++) {
                            const int rr = rbase + 16 * hh + 8 * s + rt;
                            if (rr >= M) continue;
                            float *dst = C + (size_t)rr * N + n0 + c0 + ct;
#pragma unroll
                            for (int k = 0; k < 4; k++) {
                                float2 o = make_float2(__uint_as_float(v[hh][4 * k + 2 * s]), __uint_as_float(v[hh][4 * k + 2 * s + 1]));
                                if constexpr (EPI == TC_EPI_RES)
                                    o = make_float2(__fmaf_rn(sc, o.x, r[hh][s][k].x), __fmaf_rn(sc, o.y, r[hh][s][k].y));
                                *reinterpret_cast<float2 *>(dst + 8 * k) = o;
                            }
                        }
                }
            }
            // The accumulator is drained: the MMAs may fill it again.
            tc_fence_before();
            if constexpr (CG == 2) {  // the epilogue warps together, then one arrival for the CTA
                asm volatile("bar.sync 2, %0;" ::"n"(tc_epi_warps<CG>() * 32) : "memory");
                if (warp == 2 && lane == 0) mbar_arrive_remote(acc_empty(acc), 0);
            } else {
                mbar_arrive(acc_empty(acc));
            }
        }
    }
    tc_fence_before();
    if constexpr (CG == 2) {
        cluster_sync();  // the pair's MMAs and copies into either CTA are done
        if (warp == 1)
            asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)(2 * BN))
                         : "memory");
    } else {
        __syncthreads();
        if (warp == 1)
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)(2 * BN))
                         : "memory");
    }
}

// ---- host -------------------------------------------------------------------------------------

template <int BN, int EPI = TC_EPI_F32, int CG = 1>
static cudaError_t launch_tc(const void *a, const void *b, void *c, int M, int N, int K, uint32_t *err,
                             cudaStream_t s, bool b_const, const EpiArgs &re = EpiArgs{}, int parts = 1) {
    using L = TcLayout<BN, CG>;
    CUtensorMap ma, mb;
    // The SiLU tile's B is two boxes (gate rows, up rows), one in each CTA of a pair.
    const int b_box = (EPI == TC_EPI_SILU || CG == 2) ? BN / 2 : BN;
    if (!make_map_bf16(&ma, a, (uint64_t)M, (uint64_t)K, TC_BM) || !make_map_bf16(&mb, b, (uint64_t)N, (uint64_t)K, b_box))
        return cudaErrorInvalidValue;
    auto kern = gemm_tc_kernel<BN, EPI, CG>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int tiles = ((M + TC_BM * CG - 1) / (TC_BM * CG)) * (N / BN) * parts;
    const int units = sms / CG;  // CTAs, or pairs of them
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(CG * (tiles < units ? tiles : units));
    cfg.blockDim = dim3(tc_threads<CG>());
    cfg.dynamicSmemBytes = (size_t)L::SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = CG;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = CG == 2 ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, ma, mb, c, M, N, K, err, re, (int)b_const, parts);
}

// Tiles of 256 rows for a pair of CTAs when the launch has the rows for it (the prefill's).
constexpr int TC_PAIR_MIN_ROWS = 256;

cudaError_t launch_gemm(const tg_params &p, const void *a, const void *b, float *c, uint32_t *err,
                        cudaStream_t s) {
    const int M = (int)p.m, N = (int)p.n, K = (int)p.k;
    if (M <= 0 || N <= 0 || K <= 0) return cudaErrorInvalidValue;
    if (p.dtype != TG_BF16) {
        if (p.parts > 1) return cudaErrorInvalidValue;
        dim3 grid((N + 63) / 64, (M + 63) / 64);
        gemm_f32_kernel<<<grid, 256, 0, s>>>(M, N, K, (const float *)a, (const float *)b, c);
        return cudaGetLastError();
    }
    if (K % TC_BK != 0) return cudaErrorInvalidValue;
    const bool b_const = (p.flags & 1) != 0;
    const int parts = p.parts > 1 ? (int)p.parts : 1;
    if (K % (TC_BK * parts) != 0) return cudaErrorInvalidValue;
    // Narrow tiles (flags bit 1, a batched decode step's few rows) and parts of K: more blocks
    // stream the weights. Both are the caller's choice, not the rows': a row's sums do not depend
    // on how many rows a launch takes.
    if (p.flags & 2) {
        if (N % 64 == 0) return launch_tc<64>(a, b, c, M, N, K, err, s, b_const, EpiArgs{}, parts);
        return cudaErrorInvalidValue;
    }
    if (parts > 1) {
        if (N % 256 == 0) return launch_tc<256>(a, b, c, M, N, K, err, s, b_const, EpiArgs{}, parts);
        if (N % 128 == 0) return launch_tc<128>(a, b, c, M, N, K, err, s, b_const, EpiArgs{}, parts);
        return launch_tc<64>(a, b, c, M, N, K, err, s, b_const, EpiArgs{}, parts);
    }
    if (N % 256 == 0 && M >= TC_PAIR_MIN_ROWS) return launch_tc<256, TC_EPI_F32, 2>(a, b, c, M, N, K, err, s, b_const);
    if (N % 256 == 0) return launch_tc<256>(a, b, c, M, N, K, err, s, b_const);
    if (N % 128 == 0) return launch_tc<128>(a, b, c, M, N, K, err, s, b_const);
    if (N % 64 == 0) return launch_tc<64>(a, b, c, M, N, K, err, s, b_const);
    return cudaErrorInvalidValue;
}

cudaError_t launch_gemm_qkv_rope(const tg_params &p, const void *a, const void *b, const uint32_t *at,
                                 const float *cosv, const float *sinv, void *q, void *kc, void *vc, uint32_t *err,
                                 cudaStream_t s) {
    const int M = (int)p.m, N = (int)p.n, K = (int)p.k;
    if (p.dtype != TG_BF16 || M <= 0 || N % 256 || K % TC_BK || 256 % p.head_dim ||
        N != (int)((p.heads + 2 * p.kv_heads) * p.head_dim) || p.rows != p.m)
        return cudaErrorInvalidValue;
    EpiArgs re{p, at, cosv, sinv, (bf16 *)q, (bf16 *)kc, (bf16 *)vc, nullptr};
    // A tile holds whole heads; narrow tiles (flags bit 1, a batched decode step) one head each, so
    // that more blocks stream the weights.
    if ((p.flags & 2) && p.head_dim == 64) return launch_tc<64, TC_EPI_ROPE>(a, b, nullptr, M, N, K, err, s, true, re);
    if (M >= TC_PAIR_MIN_ROWS) return launch_tc<256, TC_EPI_ROPE, 2>(a, b, nullptr, M, N, K, err, s, true, re);
    return launch_tc<256, TC_EPI_ROPE>(a, b, nullptr, M, N, K, err, s, true, re);
}

cudaError_t launch_gemm_residual(const tg_params &p, const void *a, const void *b, const float *res, float *out,
                                 uint32_t *err, cudaStream_t s) {
    const int M = (int)p.m, N = (int)p.n, K = (int)p.k;
    if (p.dtype != TG_BF16 || M <= 0 || N % 64 || K % TC_BK || p.parts > 1) return cudaErrorInvalidValue;
    EpiArgs re{};
    re.p = p;
    re.res = res;
    const bool b_const = (p.flags & 1) != 0;
    if (N % 256 == 0 && M >= TC_PAIR_MIN_ROWS) return launch_tc<256, TC_EPI_RES, 2>(a, b, out, M, N, K, err, s, b_const, re);
    if (N % 256 == 0) return launch_tc<256, TC_EPI_RES>(a, b, out, M, N, K, err, s, b_const, re);
    if (N % 128 == 0) return launch_tc<128, TC_EPI_RES>(a, b, out, M, N, K, err, s, b_const, re);
    return launch_tc<64, TC_EPI_RES>(a, b, out, M, N, K, err, s, b_const, re);
}

cudaError_t launch_gemm_silu(const tg_params &p, const void *a, const void *b, void *out, uint32_t *err,
                             cudaStream_t s) {
    const int M = (int)p.m, N = (int)p.n, K = (int)p.k;
    if (p.dtype != TG_BF16 || M <= 0 || N % 256 || K % TC_BK) return cudaErrorInvalidValue;
    // Narrow tiles (flags bit 1, a batched decode step): 32 outputs a tile, four times the blocks.
    if (p.flags & 2) return launch_tc<64, TC_EPI_SILU>(a, b, out, M, N, K, err, s, true);
    if (M >= TC_PAIR_MIN_ROWS) return launch_tc<256, TC_EPI_SILU, 2>(a, b, out, M, N, K, err, s, true);
    return launch_tc<256, TC_EPI_SILU>(a, b, out, M, N, K, err, s, true);
}

}  // namespace tg
