// Device helpers shared by the CARE-KV kernels.
//
// Numerics follow torch CPU semantics of the reference exactly where the
// reference's results are integers or bytes (codes, scales, packed rows,
// slot payloads): every op on an fp16 / bf16 value is computed in fp32 with
// IEEE division / multiplication (explicit __f*_rn intrinsics, so nvcc
// never contracts them into an FMA) and rounded back to the storage dtype
// with round-to-nearest-even.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/carekv_b200.h"

namespace carekv {

constexpr int kPage = 16;            // tokens per page (the only size built)
constexpr int kErrPageOverflow = 1;  // error_flag bit: page beyond max_pages
constexpr int kErrBadState = 2;      // error_flag bit: inconsistent page state

// ───────────────────────── dtype conversions ─────────────────────────
__device__ __forceinline__ float f16_bits_to_f32(uint16_t b) {
  return __half2float(__ushort_as_half(b));
}
__device__ __forceinline__ uint16_t f32_to_f16_bits(float x) {
  return __half_as_ushort(__float2half_rn(x));
}
__device__ __forceinline__ float f16r(float x) { return __half2float(__float2half_rn(x)); }
__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Round an fp32 value to activation dtype `dt`, returned as fp32.
__device__ __forceinline__ float rnd(float x, int dt) {
  if (dt == CAREKV_F16) return f16r(x);
  if (dt == CAREKV_BF16) return bf16r(x);
  return x;
}

// clamp(min=1e-8) lower bound as torch converts the scalar to the tensor dtype.
__device__ __forceinline__ float clamp_lo(int dt) {
  if (dt == CAREKV_F16) return 0.0f;  // 1e-8 underflows to +0 in fp16
  if (dt == CAREKV_BF16) return bf16r(1e-8f);
  return 1e-8f;
}

__device__ __forceinline__ float load_act(const void* p, int64_t i, int dt) {
  if (dt == CAREKV_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  if (dt == CAREKV_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ void store_act(void* p, int64_t i, float v, int dt) {
  if (dt == CAREKV_F16) reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  else if (dt == CAREKV_BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else reinterpret_cast<float*>(p)[i] = v;
}

// float -> int8 code the way torch casts after round().clamp(): NaN -> 0.
__device__ __forceinline__ int8_t to_code(float v) {
  if (v != v) return 0;
  return static_cast<int8_t>(static_cast<int>(v));
}

// ───────────────────────── base quantizer ─────────────────────────
// One group of `g` values (exact in dtype dt): scale and codes
// (quantizer.py:31-64).  qmax = 2^(bits-1)-1.
__device__ __forceinline__ float group_scale(float max_abs, int qmax, int dt) {
  float m = fmaxf(max_abs, clamp_lo(dt));
  return rnd(__fdiv_rn(m, static_cast<float>(qmax)), dt);
}
__device__ __forceinline__ int8_t quant_code(float x, float scale, int qmax, int dt) {
  float t = rnd(__fdiv_rn(x, scale), dt);
  if (t != t) return 0;  // torch's clamp keeps NaN (0/0 on an all-zero fp16 group); int8 cast -> 0
  t = rintf(t);
  t = fminf(fmaxf(t, static_cast<float>(-qmax - 1)), static_cast<float>(qmax));
  return static_cast<int8_t>(static_cast<int>(t));
}
// ───────────────────────── KIVI-style base (kivi_helpers.py:35-59) ─────────
// scale = amax / qmax rounded to dt, then clamp(min=1e-8) in dt.  A scale of
// 0 (an all-zero fp16 slice, where the clamp bound underflows to 0) makes the
// reference's codes 0/0 = NaN and its x_hat NaN; it is kept as a NaN scale so
// code * scale reads back NaN the same way.
__device__ __forceinline__ float kivi_scale(float amax, int qmax, int dt) {
  const float s = fmaxf(rnd(__fdiv_rn(amax, static_cast<float>(qmax)), dt), clamp_lo(dt));
  return s == 0.f ? __int_as_float(0x7fc00000) : s;
}
// clamp(round(rnd(x / scale)), -qmax - 1, qmax) with the quotient rounded to
// dt as torch divides in dt; a NaN quotient (zero scale) gives code 0.
__device__ __forceinline__ int kivi_code_dt(float x, float scale, int qmax, int dt) {
  float t = rintf(rnd(__fdiv_rn(x, scale), dt));
  if (t != t) return 0;
  return static_cast<int>(fminf(fmaxf(t, static_cast<float>(-qmax - 1)), static_cast<float>(qmax)));
}
// x_hat = code * scale in dt (NaN scale -> NaN)
__device__ __forceinline__ float kivi_hat(int code, float scale, int dt) {
  return rnd(__fmul_rn(static_cast<float>(code), scale), dt);
}

// dequantize: code * scale in fp32, rounded to the scale dtype.
__device__ __forceinline__ float dequant(int code, float scale, int dt) {
  return rnd(__fmul_rn(static_cast<float>(code), scale), dt);
}

// ───────────────────────── packed rows ─────────────────────────
__host__ __device__ __forceinline__ int row_bytes(int D, int bits) {
  return bits == 2 ? D / 4 : (bits == 3 ? D * 3 / 8 : D / 2);
}

// code at channel c of a packed row (quantizer.py:267-301, 327-343)
__device__ __forceinline__ int unpack_code(const uint8_t* row, int c, int bits) {
  if (bits == 3) {
    const uint8_t* w = row + 3 * (c >> 3);
    uint32_t word = w[0] | (uint32_t(w[1]) << 8) | (uint32_t(w[2]) << 16);
    int v = (word >> (3 * (c & 7))) & 7;
    return v >= 4 ? v - 8 : v;
  } else if (bits == 2) {
    int v = (row[c >> 2] >> (2 * (c & 3))) & 3;
    return v >= 2 ? v - 4 : v;
  } else {
    int v = (row[c >> 1] >> (4 * (c & 1))) & 15;
    return v >= 8 ? v - 16 : v;
  }
}

// byte j of a packed row from its codes (quantizer.py:257-324)
__device__ __forceinline__ uint8_t pack_byte(const int8_t* codes, int j, int bits) {
  if (bits == 3) {
    int w = j / 3, b = j % 3;
    uint32_t word = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) word |= (uint32_t(codes[8 * w + i]) & 7u) << (3 * i);
    return static_cast<uint8_t>((word >> (8 * b)) & 0xFF);
  } else if (bits == 2) {
    uint32_t v = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) v |= (uint32_t(codes[4 * j + i]) & 3u) << (2 * i);
    return static_cast<uint8_t>(v);
  } else {
    return static_cast<uint8_t>((uint32_t(codes[2 * j]) & 15u) | ((uint32_t(codes[2 * j + 1]) & 15u) << 4));
  }
}

// ───────────────────────── base scales ─────────────────────────
// Read one stored base scale as the fp16 value the reference dequantizes
// with (cache.py:713-718): int8 mode fp16(code*master), otherwise the stored
// scale cast to fp16.
__device__ __forceinline__ float read_scale(const void* base, int64_t i, int mode, float master) {
  switch (mode) {
    case CAREKV_SCALE_INT8:
      return f16r(__fmul_rn(static_cast<float>(reinterpret_cast<const int8_t*>(base)[i]), master));
    case CAREKV_SCALE_F16:
      return __half2float(reinterpret_cast<const __half*>(base)[i]);
    case CAREKV_SCALE_BF16:
      return f16r(__bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[i]));
    default:
      return f16r(reinterpret_cast<const float*>(base)[i]);
  }
}

// Store a raw (non-int8) scale in the scale dtype (cache.py:605-606).
__device__ __forceinline__ void write_raw_scale(void* base, int64_t i, int mode, float s) {
  if (mode == CAREKV_SCALE_F16) reinterpret_cast<__half*>(base)[i] = __float2half_rn(s);
  else if (mode == CAREKV_SCALE_BF16) reinterpret_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(s);
  else reinterpret_cast<float*>(base)[i] = s;
}

// int8 scale code against a master (cache.py:601-602, 692-693)
__device__ __forceinline__ int8_t int8_scale_code(float s, float master) {
  float t = __fdiv_rn(s, master);
  if (t != t) return 0;  // 0/0 with a zero master: NaN -> int8 0 as in torch
  t = rintf(t);
  t = fminf(fmaxf(t, -128.0f), 127.0f);
  return static_cast<int8_t>(static_cast<int>(t));
}

// ───────────────────────── 4-bit residual slots ─────────────────────────
__device__ __forceinline__ int nibble_code(float x, float s) {
  float t = rintf(__fdiv_rn(x, s));
  t = fminf(fmaxf(t, -8.0f), 7.0f);
  return static_cast<int>(t);
}
// ───────────── quotients through a reciprocal (page store hot loop) ─────────────
// RN(x / s) from r = RN(1 / s): q = RN(x r), the remainder x - q s exact by
// FMA, then RN(q + (x - q s) r) -- Markstein's correction (P. Markstein,
// IBM J. Res. Dev. 34(1), 1990; Muller et al., Handbook of Floating-Point
// Arithmetic, the division theorem with a correctly rounded reciprocal),
// exact while the remainder does not underflow.  The codes below use it
// only where that holds: quantizer quotients |x / s| <= 16 with s an fp16
// value or a bf16 value >= 1e-9 (the quantizer's scales), and 4-bit slot
// quotients |R / s4| <= 8 with s4 >= 1e-8 / 7; checked against __fdiv_rn
// over every fp16 (x, s) pair and every bf16 pair with s >= 1e-9.
__device__ __forceinline__ float div_by_recip(float x, float s, float r) {
  const float q = __fmul_rn(x, r);
  return __fmaf_rn(__fmaf_rn(-q, s, x), r, q);
}
// quant_code(x, scale) with rcp = __frcp_rn(scale)
__device__ __forceinline__ int quant_code_r(float x, float scale, float rcp, int qmax, int dt) {
  float t = rnd(div_by_recip(x, scale, rcp), dt);
  if (t != t) return 0;  // 0/0 on an all-zero fp16 group (rcp = inf): NaN -> 0 as quant_code
  t = rintf(t);
  t = fminf(fmaxf(t, static_cast<float>(-qmax - 1)), static_cast<float>(qmax));
  return static_cast<int>(t);
}
// nibble_code(x, s) with rcp = __frcp_rn(s)
__device__ __forceinline__ int nibble_code_r(float x, float s, float rcp) {
  const float t = rintf(div_by_recip(x, s, rcp));
  return static_cast<int>(fminf(fmaxf(t, -8.0f), 7.0f));
}
__device__ __forceinline__ float unpack_nibble(const uint8_t* payload, int i, float scale) {
  int v = (payload[i >> 1] >> (4 * (i & 1))) & 15;
  if (v > 7) v -= 16;
  return __fmul_rn(static_cast<float>(v), scale);
}

// ───────────────────────── reductions ─────────────────────────
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ───────────────────────── arena indexing ─────────────────────────
struct Dims {
  int L, H, P, D, R, G, C, NV, SK, SV, kslot_bytes, vslot_bytes, sketch;
  int bits, gsize, kcg, vtb, scale_mode;
  int scale_elem;  // bytes per stored base scale
  int kivi;        // 1: KIVI base (per-channel K / per-token V scales, fp16 K window)
  int W;           // KIVI: window pages of decode-appended fp16 K rows

  __host__ __device__ int64_t lhp(int b, int l, int h) const {
    return (static_cast<int64_t>(b) * L + l) * H + h;
  }
  __host__ __device__ int64_t page(int b, int l, int h, int p) const {
    return lhp(b, l, h) * P + p;
  }
};

// every field except the three ratios G, C, NV
__host__ __device__ inline Dims make_dims_shared(const carekv_config_t& c) {
  Dims d;
  d.L = c.num_layers;
  d.H = c.num_kv_heads;
  d.P = c.max_pages;
  d.D = c.head_dim;
  d.bits = c.base_bits;
  d.R = row_bytes(c.head_dim, c.base_bits);
  d.gsize = c.group_size;
  d.kcg = c.k_channel_group;
  d.vtb = c.v_token_block;
  d.SK = c.k_slots_per_page;
  d.SV = c.v_slots_per_page;
  d.kslot_bytes = kPage * c.k_channel_group / 2;
  d.vslot_bytes = c.v_token_block * c.head_dim / 2;
  d.sketch = c.sketch_dim;
  d.scale_mode = c.scale_mode;
  d.scale_elem = c.scale_mode == CAREKV_SCALE_INT8 ? 1 : (c.scale_mode == CAREKV_SCALE_F32 ? 4 : 2);
  d.kivi = c.base_kind == CAREKV_BASE_KIVI;
  d.W = d.kivi ? c.kivi_window_pages : 0;
  return d;
}
__host__ __device__ inline Dims make_dims(const carekv_config_t& c) {
  Dims d = make_dims_shared(c);
  d.G = c.head_dim / c.group_size;
  d.C = c.head_dim / c.k_channel_group;
  d.NV = kPage / c.v_token_block;
  return d;
}

// make_dims with shifts for the ratios of power-of-two sizes (head_dim,
// group size, K channel group, V token block: checked at cache init).
__device__ inline Dims make_dims_p2(const carekv_config_t& c) {
  Dims d = make_dims_shared(c);
  const int lgD = __ffs(c.head_dim) - 1;
  d.G = 1 << (lgD - (__ffs(c.group_size) - 1));
  d.C = 1 << (lgD - (__ffs(c.k_channel_group) - 1));
  d.NV = kPage >> (__ffs(c.v_token_block) - 1);
  return d;
}

}  // namespace carekv
