// Warp-level tensor-core building blocks (mma.sync m16n8k16 with bf16 operands, ldmatrix, cp.async)
// shared by the prefill's mma.sync flash attention and the batched decoder's split attention.
#pragma once

#include "tg_common.cuh"

namespace tg {

namespace fa {

constexpr int KT = 64;  // keys per tile
constexpr int PAD = 8;  // bf16 elements of padding per shared row (ldmatrix without bank conflicts)

TG_DEVICE void cp_async16(void *smem, const void *gmem, bool valid) {
    const uint32_t dst = smem_u32(smem);
    const int bytes = valid ? 16 : 0;  // zero-fill when invalid
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(gmem), "r"(bytes) : "memory");
}
TG_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
TG_DEVICE void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

TG_DEVICE void ldmatrix_x4(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
TG_DEVICE void ldmatrix_x4_trans(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
TG_DEVICE void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// x0, x1 as bf16 pairs hi and lo with hi + lo = x to about 16 bits (hi rounded, lo the rest rounded).
TG_DEVICE void split_pack(float x0, float x1, uint32_t &hi, uint32_t &lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
    const float h0 = __low2float(h), h1 = __high2float(h);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(__fsub_rn(x0, h0), __fsub_rn(x1, h1));
    lo = *reinterpret_cast<const uint32_t *>(&l);
}
TG_DEVICE uint32_t pack_bf16(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&v);
}

}  // namespace fa

}  // namespace tg
