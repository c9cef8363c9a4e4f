// Inline-PTX helpers shared by the decode kernels (sm_100a): mbarrier +
// bulk-copy staging with bounded waits, the m16n8k16 fp16 tensor-core MMA and
// half2 bit tricks for exact low-bit dequantization.
#pragma once
#include <cuda_fp16.h>
#include <cstdint>

namespace carekv {

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
// Bulk copy global -> this CTA's shared memory, completion counted on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}
// L2 eviction policies: streamed data that is read once, and results the
// next kernel reads back.
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint64_t l2_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// bulk_g2s with an L2 eviction policy
__device__ __forceinline__ void bulk_g2s_pol(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(pol)
      : "memory");
}
// 8-byte global store with an L2 eviction policy
__device__ __forceinline__ void st_f2_pol(float* p, float x, float y, uint64_t pol) {
  asm volatile("st.global.L2::cache_hint.v2.f32 [%0], {%1, %2}, %3;" ::"l"(p), "f"(x), "f"(y), "l"(pol) : "memory");
}
// One arrival (release, CTA scope) on an mbarrier.
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false after ~2^31 cycles (about a second) without completion.
// The clock is read only when the first test fails.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > (1ll << 31)) return false;
  }
  return true;
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

// D += A . B, m16n8k16, fp16 inputs, fp32 accumulation.
__device__ __forceinline__ void mma_f16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t h2sub(uint32_t a, uint32_t b) {
  __half2 r = __hsub2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t h2mul(uint32_t a, uint32_t b) {
  __half2 r = __hmul2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  __half2 r = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) { return __byte_perm(a, b, sel); }

// A 3-bit two's-complement field f at mantissa bit s of an fp16 half, with
// the half's exponent set to 25 - s and bit 2 of the field flipped by the
// XOR, reads as 2^(10-s) + (f ^ 4) = 2^(10-s) + code + 4; the same key read
// as fp16 is 2^(10-s) + 4, so one HSUB2 leaves the code exactly.
__host__ __device__ constexpr uint32_t i3_key(int s) {
  return ((25u - static_cast<uint32_t>(s)) << 10) | (4u << s);
}
__host__ __device__ constexpr uint32_t i3_key2(int s_lo, int s_hi) { return i3_key(s_lo) | (i3_key(s_hi) << 16); }
__host__ __device__ constexpr uint32_t i3_mask2(int s_lo, int s_hi) {
  return (7u << s_lo) | (7u << (16 + s_hi));
}
// exact half2 of (code_lo, code_hi) * sig2 from a register holding field lo at
// bit s_lo of its low half and field hi at bit s_hi of its high half
template <int SL, int SH>
__device__ __forceinline__ uint32_t i3_pair(uint32_t t, uint32_t sig2) {
  return h2mul(h2sub((t & i3_mask2(SL, SH)) ^ i3_key2(SL, SH), i3_key2(SL, SH)), sig2);
}

// Two int8 scale codes (b_lo, b_hi, zero-extended bytes at bits 0 and 16)
// times an fp16 master (duplicated in m2) -> half2 of fp16(code * master),
// rounded once like fp16(float(code) * master).  1024 + (b ^ 0x80) - 1152 = b.
__device__ __forceinline__ uint32_t i8_scale_pair(uint32_t bytes, uint32_t m2) {
  const uint32_t x = (bytes ^ 0x00800080u) | 0x64006400u;
  return h2mul(h2sub(x, 0x64806480u), m2);
}

// Byte k of w (two 4-bit two's-complement codes, even channel in the low
// nibble) -> half2 of the exact codes.  The low nibble goes to mantissa bit 0
// of the low half (value 1024 + u), the high nibble to bit 4 of the high half
// (value 64 + u); the XOR of bit 3 turns two's complement into u = code + 8
// and the same key read as fp16 is the offset removed by the subtraction.
__device__ __forceinline__ uint32_t nib_pair(uint32_t w, int k) {
  const uint32_t y = __byte_perm(w, 0u, 0x4040u | (static_cast<uint32_t>(k) * 0x0101u));
  const uint32_t key = 0x54806408u;
  const uint32_t x = (y & 0x00F0000Fu) ^ key;
  return h2sub(x, key);
}

}  // namespace carekv
