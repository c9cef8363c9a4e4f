// Prefill page store, one warp per page (kernel K1, prefill form).
//
// Replaces, for the uniform per-group base with fp16 / bf16 inputs:
//   layer.py:204-334      _write_pages_for_kv_head (prefill pages)
//   cache.py:592-640      write_base: codes, packed rows, int8 page scales
//   residual_store.py:239-464  ResidualStoreManager.process_page
//
// The same outputs as page_store_kernel<0> (store.cu), laid out for the
// prefill rate: one warp owns one 16-row page and lane l owns half of row
// l/2 (channels (l&1)*D/2 .. +D/2) of both K and V, held in registers.  A
// quantization group (D/4, D/2 or D channels) lies inside one lane or one
// lane pair, so group maxima, scale codes and the packed row bytes are
// lane-local; page-wide quantities (int8 master, candidate error norms and
// maxima, the V_hat norm) are warp shuffles, and the 4-bit payload of a
// candidate is formed only when the page keeps it.  No shared memory and no
// CTA barrier: warps run their pages independently.
//
// Arithmetic per element is the store kernel's (common.cuh: group_scale,
// quant_code, dequant, int8_scale_code, nibble_code), in forms that give
// the same values: code quotients through a correctly rounded reciprocal
// (div_by_recip, the IEEE quotient on these operands), X_hat = code * s and
// R = X - X_hat as one rounding in fp16 / bf16 pair arithmetic (the fp32
// product and difference are exact before the store kernel rounds them to
// the dtype).  Codes, scales, masters and payloads are therefore
// bit-identical to it for finite inputs (a NaN input row gets the clamped
// code instead of 0); the error norms and the
// V_hat norm accumulate in a different fp32 order (per-lane partial sums,
// then a butterfly), as the store kernel's order differs from the
// reference's own.
#include "common.cuh"
#include "internal.h"

namespace carekv {
namespace pstore {

constexpr int kWarps = 8;   // warps per CTA: a K and a V warp per page

// 2-byte activation pair -> two floats
template <int DT>
__device__ __forceinline__ float2 unpack2(uint32_t w) {
  if (DT == CAREKV_BF16) return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  const __half2 h = *reinterpret_cast<const __half2*>(&w);
  return __half22float2(h);
}
// The larger magnitude of a lane-wise 16-bit max of |x| bits (x & 0x7fff
// per half: magnitudes of finite fp16 / bf16 values order like their bits)
template <int DT>
__device__ __forceinline__ float abs_pair_max(uint32_t mu) {
  mu = max(mu & 0xffffu, mu >> 16);
  return DT == CAREKV_BF16 ? __uint_as_float(mu << 16) : __half2float(__ushort_as_half(static_cast<unsigned short>(mu)));
}

// (lo, hi) -> dt pair with round to nearest even (lo in the low half)
template <int DT>
__device__ __forceinline__ uint32_t cvt_pair(float lo, float hi) {
  uint32_t d;
  if (DT == CAREKV_BF16) asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  else asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}
// lane-wise a * b and a - b of dt pairs, one rounding to nearest even each
template <int DT>
__device__ __forceinline__ uint32_t mul_pair(uint32_t a, uint32_t b) {
  uint32_t d;
  if (DT == CAREKV_BF16) asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  else asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
template <int DT>
__device__ __forceinline__ uint32_t sub_pair(uint32_t a, uint32_t b) {
  uint32_t d;
  if (DT == CAREKV_BF16) asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  else asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Store n bytes (n = 4, 8, 12, 16, 24 or 32) of w[] at dst, in the widest
// words the alignment of n allows (dst is aligned to the same width).
template <int NB>
__device__ __forceinline__ void store_bytes(uint8_t* dst, const uint32_t (&w)[(NB + 3) / 4]) {
  if constexpr (NB % 16 == 0) {
#pragma unroll
    for (int i = 0; i < NB / 16; ++i)
      reinterpret_cast<uint4*>(dst)[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
  } else if constexpr (NB % 8 == 0) {
#pragma unroll
    for (int i = 0; i < NB / 8; ++i) reinterpret_cast<uint2*>(dst)[i] = make_uint2(w[2 * i], w[2 * i + 1]);
  } else {
#pragma unroll
    for (int i = 0; i < NB / 4; ++i) reinterpret_cast<uint32_t*>(dst)[i] = w[i];
  }
}

// Page-pair scratch: the candidates' error norms and 4-bit scales, so that
// the K and V warps of a page rank them together.
struct PairSmem {
  float e[32];
  float s4[32];
};

// GSEL: quantization group = D/4 (0: two groups per lane), D/2 (1: one
// group per lane) or D (2: one group per lane pair).  kind 0: the K warp of
// a page, 1: its V warp -- one code path for both, so the two warps of a
// page run the same instructions.
template <int D, int BITS, int GSEL, int DT>
__device__ __forceinline__ void store_half(const carekv_config_t& cfg, const carekv_cache_t& cache, int layer,
                                           const void* __restrict__ Xin, int T, int seq_begin,
                                           const carekv_store_params_t& prm, int in_H, int64_t gw, int pair,
                                           int kind, PairSmem& ps) {
  constexpr int NE = D / 2;            // elements per lane
  constexpr int NW = NE / 2;           // packed 2-byte pairs per lane
  constexpr int GPL = GSEL == 0 ? 2 : 1;
  constexpr int GL = NE / GPL;         // elements of one lane-local group
  constexpr int G = GSEL == 0 ? 4 : (GSEL == 1 ? 2 : 1);   // groups per row
  constexpr int CPL = NE / 32;         // K residual candidates (32 channels) per lane
  constexpr int C = D / 32;
  constexpr int HB = NE * BITS / 8;    // packed bytes of a half row
  constexpr int R = D * BITS / 8;
  constexpr int qmax = (1 << (BITS - 1)) - 1;
  constexpr int dt = DT;

  const Dims d = make_dims(cfg);
  const int lane = threadIdx.x & 31;
  const int r = lane >> 1, hf = lane & 1;
  const int n_new = (T + kPage - 1) / kPage;
  const int pi = static_cast<int>(gw % n_new);
  const int sh = static_cast<int>(gw / n_new);
  const int h = sh % d.H, s = sh / d.H;
  const int64_t lhp = d.lhp(seq_begin + s, layer, h);
  const int p = cache.num_pages[lhp] + pi;
  if (p >= d.P) {
    if (lane == 0 && kind == 0) atomicOr(cache.error_flag, kErrPageOverflow);
    return;   // both warps of the pair leave before their barrier
  }
  const int64_t pg = lhp * d.P + p;
  const int t0 = pi * kPage;
  const int nv = min(kPage, T - t0);
  const bool live = r < nv;

  // ── the lane's half row, every load issued first (rows past the valid
  // count are zero, layer.py:262-271) ──
  uint32_t x[NW];
  {
    const int64_t off = (((static_cast<int64_t>(s) * in_H + h) * T + t0 + r) * D + hf * NE) * 2;
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(Xin) + off);
#pragma unroll
    for (int i = 0; i < NW / 4; ++i) {
      uint4 a = make_uint4(0u, 0u, 0u, 0u);
      if (live) a = __ldg(src + i);
      x[4 * i] = a.x; x[4 * i + 1] = a.y; x[4 * i + 2] = a.z; x[4 * i + 3] = a.w;
    }
  }

  // ── group scales (quantizer.py:31-64; max is order-free) ──
  // |x| of fp16 / bf16 values orders like the integer bits & 0x7fff, so the
  // group maximum is taken on the packed pairs (16-bit lane-wise max)
  float m[GPL];
#pragma unroll
  for (int j = 0; j < GPL; ++j) {
    uint32_t mu = 0u;
#pragma unroll
    for (int w = j * (NW / GPL); w < (j + 1) * (NW / GPL); ++w) mu = __vmaxu2(mu, x[w] & 0x7fff7fffu);
    m[j] = abs_pair_max<DT>(mu);
  }
  if (GSEL == 2) m[0] = fmaxf(m[0], __shfl_xor_sync(0xffffffffu, m[0], 1));
  float sc[GPL], rcp[GPL], rs[GPL];
#pragma unroll
  for (int j = 0; j < GPL; ++j) {
    sc[j] = group_scale(m[j], qmax, dt);
    // a zero scale (an all-zero fp16 group, where the clamp bound underflows)
    // takes reciprocal 0: its x are all 0 and so are its codes, as the
    // reference's 0/0 -> NaN -> int8 0
    rcp[j] = sc[j] > 0.f ? __frcp_rn(sc[j]) : 0.f;
  }
  // page scales (cache.py:592-606): int8 codes against the page master, or
  // the raw scale; rs = the scale as read back (fp16 value)
  void* sdst = kind ? cache.v_scale : cache.k_scale;
  const int64_t srow = (pg * kPage + r) * G + (GSEL == 0 ? 2 * hf : (GSEL == 1 ? hf : 0));
  const bool writer = GSEL != 2 || hf == 0;
  if (d.scale_mode == CAREKV_SCALE_INT8) {
    float mx = 0.f;
#pragma unroll
    for (int j = 0; j < GPL; ++j) mx = fmaxf(mx, fabsf(sc[j]));
    mx = fmaxf(warp_max(mx), clamp_lo(dt));
    const uint16_t mb = f32_to_f16_bits(__fdiv_rn(mx, 127.0f));
    const float master = f16_bits_to_f32(mb);
    if (lane == 0) (kind ? cache.v_master : cache.k_master)[pg] = mb;
    uint32_t c8w = 0u;
#pragma unroll
    for (int j = 0; j < GPL; ++j) {
      const int8_t c8 = int8_scale_code(sc[j], master);
      rs[j] = f16r(__fmul_rn(static_cast<float>(c8), master));
      c8w |= static_cast<uint32_t>(static_cast<uint8_t>(c8)) << (8 * j);
    }
    int8_t* sd = reinterpret_cast<int8_t*>(sdst) + srow;
    if (GPL == 2) *reinterpret_cast<uint16_t*>(sd) = static_cast<uint16_t>(c8w);
    else if (writer) *sd = static_cast<int8_t>(c8w);
  } else {
#pragma unroll
    for (int j = 0; j < GPL; ++j) {
      if (writer) write_raw_scale(sdst, srow + j, d.scale_mode, sc[j]);
      rs[j] = d.scale_mode == CAREKV_SCALE_BF16 ? f16r(bf16r(sc[j])) : f16r(sc[j]);
    }
  }

  // ── codes, packed row bits, residual R = X - X_hat in place
  // (residual_store.py:271-285), V_hat norm ──
  constexpr int NPW = (HB + 3) / 4;
  uint32_t pk[NPW];
#pragma unroll
  for (int i = 0; i < NPW; ++i) pk[i] = 0u;
  float vn = 0.f;
  const bool vnorm = kind && live;
  // the group scales as dt pairs (exact: they are dt values), the read-back
  // V scales as fp16 pairs
  uint32_t s2[GPL], rs2[GPL];
#pragma unroll
  for (int j = 0; j < GPL; ++j) {
    s2[j] = cvt_pair<DT>(sc[j], sc[j]);
    rs2[j] = cvt_pair<CAREKV_F16>(rs[j], rs[j]);
  }
  const float lo = static_cast<float>(-qmax - 1), hi = static_cast<float>(qmax);
#pragma unroll
  for (int w = 0; w < NW; ++w) {
    const float2 f = unpack2<DT>(x[w]);
    const int j = (2 * w) / GL;
    // code = clamp(rint(dt(x / s))) (quant_code; the quotient as div_by_recip)
    const float2 qd = unpack2<DT>(cvt_pair<DT>(div_by_recip(f.x, sc[j], rcp[j]), div_by_recip(f.y, sc[j], rcp[j])));
    float t0 = rintf(qd.x), t1 = rintf(qd.y);
    if constexpr (DT != CAREKV_BF16) {
      // fp16 scales may be subnormal, their quotients above qmax; a bf16
      // scale is normal (>= clamp / qmax) and within 2^-8 of max / qmax, so
      // |x / s| <= qmax (1 + 2^-8) rounds inside [-qmax, qmax]
      t0 = fminf(fmaxf(t0, lo), hi);
      t1 = fminf(fmaxf(t1, lo), hi);
    }
    // codes 2w, 2w+1 at bits BITS*e of the half row's little-endian stream;
    // t + 1.5*2^23 holds t in two's complement in its low mantissa bits
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const uint32_t cu = __float_as_uint((u ? t1 : t0) + 12582912.0f) & ((1u << BITS) - 1u);
      const int bit = BITS * (2 * w + u);
      pk[bit / 32] |= cu << (bit % 32);
      if (bit % 32 > 32 - BITS) pk[bit / 32 + 1] |= cu >> (32 - bit % 32);
    }
    // X_hat = dt(code * s) and R = dt(X - X_hat), both one rounding in the
    // dt pair arithmetic, equal to the fp32-then-dt rounding of dequant and
    // the residual (code * s and X - X_hat are exact in fp32 here)
    const uint32_t c2 = cvt_pair<DT>(t0, t1);
    x[w] = sub_pair<DT>(x[w], mul_pair<DT>(c2, s2[j]));
    if (vnorm) {
      // V rows as stored: code * the scale as read back, in fp16
      const float2 v = unpack2<CAREKV_F16>(mul_pair<CAREKV_F16>(cvt_pair<CAREKV_F16>(t0, t1), rs2[j]));
      vn = fmaf(v.x, v.x, vn);
      vn = fmaf(v.y, v.y, vn);
    }
  }
  store_bytes<HB>((kind ? cache.v_codes : cache.k_codes) + (pg * kPage + r) * R + hf * HB, pk);

  // ── candidates (residual_store.py:290-330): mean row error norm and the
  // 4-bit scale max(|R|, 1e-8) / 7 (residual_store.py:127-136) ──
  const int ncand = C + d.NV;
  if (kind == 0) {
    // K channel groups of 32: CPL per lane, shared by the 16 lanes of a half
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
      float ss = 0.f;
      uint32_t mu = 0u;
#pragma unroll
      for (int w = 16 * j; w < 16 * j + 16; ++w) {
        const float2 f = unpack2<DT>(x[w]);
        ss = fmaf(f.x, f.x, ss);
        ss = fmaf(f.y, f.y, ss);
        mu = __vmaxu2(mu, x[w] & 0x7fff7fffu);
      }
      float mj = abs_pair_max<DT>(mu);
      float ej = live ? sqrtf(ss) : 0.f;
#pragma unroll
      for (int o = 2; o < 32; o <<= 1) {
        ej += __shfl_xor_sync(0xffffffffu, ej, o);
        mj = fmaxf(mj, __shfl_xor_sync(0xffffffffu, mj, o));
      }
      // candidate hf * CPL + j: written by lane hf (row 0)
      if (lane < 2) {
        ps.e[lane * CPL + j] = nv > 0 ? __fdiv_rn(ej, static_cast<float>(nv)) : 0.f;
        ps.s4[lane * CPL + j] = __fdiv_rn(fmaxf(mj, 1e-8f), 7.0f);
      }
    }
  } else {
    // V token blocks of vtb rows: lanes 2*vtb*b .. 2*vtb*(b+1)-1
    float ss = 0.f;
    uint32_t mu = 0u;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float2 f = unpack2<DT>(x[w]);
      ss = fmaf(f.x, f.x, ss);
      ss = fmaf(f.y, f.y, ss);
      mu = __vmaxu2(mu, x[w] & 0x7fff7fffu);
    }
    float mv = abs_pair_max<DT>(mu);
    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
    mv = fmaxf(mv, __shfl_xor_sync(0xffffffffu, mv, 1));
    float ev = live ? sqrtf(ss) : 0.f;
    for (int o = 2; o < 2 * d.vtb; o <<= 1) {
      ev += __shfl_xor_sync(0xffffffffu, ev, o);
      mv = fmaxf(mv, __shfl_xor_sync(0xffffffffu, mv, o));
    }
    const int blk = r / d.vtb;
    if ((lane & (2 * d.vtb - 1)) == 0) {
      const int tb = blk * d.vtb, t1 = min(tb + d.vtb, nv);
      ps.e[C + blk] = t1 > tb ? __fdiv_rn(ev, static_cast<float>(t1 - tb)) : 0.f;
      ps.s4[C + blk] = __fdiv_rn(fmaxf(mv, 1e-8f), 7.0f);
    }
    vn = warp_sum(vn);
    if (lane == 0) {
      cache.v_norm2[pg] = vn;
      cache.valid[pg] = nv;
    }
  }
  asm volatile("bar.sync %0, 64;" ::"r"(1 + pair) : "memory");

  // ── selection (residual_store.py:370-423), lane x = candidate x; both
  // warps rank identically and each writes its own kind's slots ──
  const bool isk = lane < C, isv = lane >= C && lane < ncand;
  const float e = (isk || isv) ? ps.e[lane] : 0.f;
  const bool pos = prm.sensitivity > 0.f && !prm.store_nothing;
  const bool elig = (isk || isv) && pos && e > 0.f;
  int rank = 0, other = 0;   // rank in its kind; merged-order predecessors of the other kind
  for (int o = 0; o < ncand; ++o) {
    const float eo = ps.e[o];
    if (!(pos && eo > 0.f) || !(isk || isv)) continue;
    if ((o < C) == isk) {
      if (eo > e || (eo == e && o < lane)) ++rank;
    } else {
      if (isk ? eo > e : eo >= e) ++other;   // a V entry precedes a K entry only with a larger error
    }
  }
  const unsigned bk = __ballot_sync(0xffffffffu, elig && isk), bv = __ballot_sync(0xffffffffu, elig && isv);
  int keep_k, keep_v;
  if (prm.joint_budget > 0) {
    const bool in = elig && rank + other < prm.joint_budget;
    keep_k = __popc(__ballot_sync(0xffffffffu, in && isk));
    keep_v = __popc(__ballot_sync(0xffffffffu, in && isv));
  } else {
    keep_k = min(__popc(bk), prm.k_budget);
    keep_v = min(__popc(bv), prm.v_budget);
  }
  keep_k = min(keep_k, d.SK);
  keep_v = min(keep_v, d.SV);
  // this warp's kind: K channel groups or V token blocks
  const bool mine = kind ? isv : isk;
  const int cap = kind ? d.SV : d.SK, c0k = kind ? C : 0;
  const bool kept = elig && mine && rank < (kind ? keep_v : keep_k);
  const unsigned km = __ballot_sync(0xffffffffu, kept);
  const int nk = __popc(km);
  int8_t* const sgrp = kind ? cache.v_slot_block : cache.k_slot_group;
  uint16_t* const sscl = kind ? cache.v_slot_scale : cache.k_slot_scale;
  int32_t* const sid = kind ? cache.v_slot_id : cache.k_slot_id;
  if (kept) {
    const int64_t sidx = pg * cap + __popc(km & ((1u << lane) - 1u));
    sgrp[sidx] = static_cast<int8_t>(lane - c0k);
    sscl[sidx] = f32_to_f16_bits(ps.s4[lane]);
    sid[sidx] = rank;  // local rank; the scan adds the arena base
  }
  if (lane >= nk && lane < cap) {
    sgrp[pg * cap + lane] = -1;
    sid[pg * cap + lane] = -1;
  }
  if (mine) (kind ? cache.v_err + pg * d.NV : cache.k_err + pg * C)[lane - c0k] = f32_to_f16_bits(e);

  // ── payloads of the kept slots, their nibbles spread over all 32 lanes ──
  if (kind == 0) {
    // K group g: value i = t*32 + c (byte i/2, low nibble = even i); lane
    // (r, hf) codes channels hf*16 .. hf*16+15 of row r, fetched from the
    // lane of row r that holds group g
    unsigned mm = km;
    for (int j = 0; j < nk; ++j) {
      const int g = __ffs(mm) - 1;
      mm &= mm - 1;
      const float s4 = ps.s4[g], r4 = __frcp_rn(s4);
      const int jj = g % CPL, src = 2 * r + g / CPL;
      uint32_t pw[2] = {0u, 0u};
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        uint32_t a0 = x[k], a1 = x[8 + k];
#pragma unroll
        for (int q = 1; q < CPL; ++q)
          if (q == jj) { a0 = x[16 * q + k]; a1 = x[16 * q + 8 + k]; }
        const uint32_t v0 = __shfl_sync(0xffffffffu, a0, src), v1 = __shfl_sync(0xffffffffu, a1, src);
        const float2 f = unpack2<DT>(hf ? v1 : v0);
        const uint32_t by = (static_cast<uint32_t>(nibble_code_r(f.x, s4, r4)) & 15u) |
                            ((static_cast<uint32_t>(nibble_code_r(f.y, s4, r4)) & 15u) << 4);
        pw[k >> 2] |= by << (8 * (k & 3));
      }
      *reinterpret_cast<uint2*>(cache.k_slot_data + (pg * d.SK + j) * d.kslot_bytes + r * 16 + hf * 8) =
          make_uint2(pw[0], pw[1]);
    }
  } else {
    // V block b: value i = (t - tb)*D + c; byte k of the block is word k of
    // its lanes 2tb, 2tb+1, ... in order
    unsigned mm = km;
    for (int j = 0; j < nk; ++j) {
      const int xc = __ffs(mm) - 1;
      mm &= mm - 1;
      const float s4 = ps.s4[xc], r4 = __frcp_rn(s4);
      const int tb = (xc - C) * d.vtb;
      uint8_t* const dst = cache.v_slot_data + (pg * d.SV + j) * d.vslot_bytes;
      if (d.vtb == 4) {
        // 8 source lanes x NW words = 32 lanes x WPL bytes
        constexpr int WPL = NW / 4;
        const int src = 2 * tb + (lane >> 2), part = lane & 3;
        uint32_t y[WPL];
#pragma unroll
        for (int w = 0; w < NW; ++w) {
          const uint32_t v = __shfl_sync(0xffffffffu, x[w], src);
          if (w / WPL == part) y[w % WPL] = v;
        }
        uint32_t pw[WPL / 4];
#pragma unroll
        for (int i = 0; i < WPL / 4; ++i) pw[i] = 0u;
#pragma unroll
        for (int k = 0; k < WPL; ++k) {
          const float2 f = unpack2<DT>(y[k]);
          const uint32_t by = (static_cast<uint32_t>(nibble_code_r(f.x, s4, r4)) & 15u) |
                              ((static_cast<uint32_t>(nibble_code_r(f.y, s4, r4)) & 15u) << 4);
          pw[k >> 2] |= by << (8 * (k & 3));
        }
        store_bytes<WPL>(dst + lane * WPL, pw);
      } else if (r >= tb && r < tb + d.vtb) {
        uint32_t pw[NW / 4];
#pragma unroll
        for (int i = 0; i < NW / 4; ++i) pw[i] = 0u;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
          const float2 f = unpack2<DT>(x[w]);
          const uint32_t by = (static_cast<uint32_t>(nibble_code_r(f.x, s4, r4)) & 15u) |
                              ((static_cast<uint32_t>(nibble_code_r(f.y, s4, r4)) & 15u) << 4);
          pw[w >> 2] |= by << (8 * (w & 3));
        }
        store_bytes<NW>(dst + ((r - tb) * D + hf * NE) / 2, pw);
      }
    }
  }
}

template <int D, int BITS, int GSEL, int DT>
__global__ void __launch_bounds__(kWarps * 32, 3) page_store_warp(carekv_config_t cfg, carekv_cache_t cache, int layer,
                                                               const void* __restrict__ Kin,
                                                               const void* __restrict__ Vin, int T, int seq_begin,
                                                               int n_seq, carekv_store_params_t prm, int in_H) {
  __shared__ PairSmem ps[kWarps / 2];
  const int warp = threadIdx.x >> 5, pair = warp >> 1, kind = warp & 1;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * (kWarps / 2) + pair;   // page of this warp pair
  if (gw >= static_cast<int64_t>(n_seq) * cfg.num_kv_heads * ((T + kPage - 1) / kPage)) return;
  store_half<D, BITS, GSEL, DT>(cfg, cache, layer, kind ? Vin : Kin, T, seq_begin, prm, in_H, gw, pair, kind,
                                ps[pair]);
}

template <int D, int BITS, int GSEL>
cudaError_t launch_dt(const carekv_config_t& cfg, const carekv_cache_t& cache, int layer, const void* K,
                      const void* V, int T, int seq_begin, int seq_count, const carekv_store_params_t& prm,
                      int in_H, cudaStream_t st) {
  const int64_t pages = static_cast<int64_t>(seq_count) * cfg.num_kv_heads * ((T + kPage - 1) / kPage);
  const unsigned blocks = static_cast<unsigned>((pages + kWarps / 2 - 1) / (kWarps / 2));
  if (prm.input_dtype == CAREKV_BF16)
    page_store_warp<D, BITS, GSEL, CAREKV_BF16><<<blocks, kWarps * 32, 0, st>>>(cfg, cache, layer, K, V, T, seq_begin,
                                                                                seq_count, prm, in_H);
  else
    page_store_warp<D, BITS, GSEL, CAREKV_F16><<<blocks, kWarps * 32, 0, st>>>(cfg, cache, layer, K, V, T, seq_begin,
                                                                               seq_count, prm, in_H);
  return cudaGetLastError();
}

template <int D, int BITS>
cudaError_t launch_gs(const carekv_config_t& cfg, const carekv_cache_t& cache, int layer, const void* K,
                      const void* V, int T, int seq_begin, int seq_count, const carekv_store_params_t& prm,
                      int in_H, cudaStream_t st) {
  if (cfg.group_size == D / 4) return launch_dt<D, BITS, 0>(cfg, cache, layer, K, V, T, seq_begin, seq_count, prm, in_H, st);
  if (cfg.group_size == D / 2) return launch_dt<D, BITS, 1>(cfg, cache, layer, K, V, T, seq_begin, seq_count, prm, in_H, st);
  return launch_dt<D, BITS, 2>(cfg, cache, layer, K, V, T, seq_begin, seq_count, prm, in_H, st);
}

template <int D>
cudaError_t launch_bits(const carekv_config_t& cfg, const carekv_cache_t& cache, int layer, const void* K,
                        const void* V, int T, int seq_begin, int seq_count, const carekv_store_params_t& prm,
                        int in_H, cudaStream_t st) {
  switch (cfg.base_bits) {
    case 2: return launch_gs<D, 2>(cfg, cache, layer, K, V, T, seq_begin, seq_count, prm, in_H, st);
    case 3: return launch_gs<D, 3>(cfg, cache, layer, K, V, T, seq_begin, seq_count, prm, in_H, st);
    default: return launch_gs<D, 4>(cfg, cache, layer, K, V, T, seq_begin, seq_count, prm, in_H, st);
  }
}

}  // namespace pstore

bool prefill_store_warp_supported(const carekv_config_t& cfg, const carekv_cache_t& cache, const void* K,
                                  const void* V, const carekv_store_params_t& prm) {
  const int D = cfg.head_dim;
  const bool al = (reinterpret_cast<uintptr_t>(K) & 15) == 0 && (reinterpret_cast<uintptr_t>(V) & 15) == 0;
  const bool gs = cfg.group_size == D / 4 || cfg.group_size == D / 2 || cfg.group_size == D;
  const bool no_sketch = cache.k_sketch == nullptr || cfg.sketch_dim == 0;
  const int vtb = cfg.v_token_block;
  return cfg.base_kind == CAREKV_BASE_UNIFORM && (D == 64 || D == 128) && gs && cfg.group_size >= 16 &&
         (cfg.base_bits >= 2 && cfg.base_bits <= 4) &&
         (prm.input_dtype == CAREKV_BF16 || prm.input_dtype == CAREKV_F16) && cfg.k_channel_group == 32 &&
         (vtb == 1 || vtb == 2 || vtb == 4 || vtb == 8 || vtb == 16) && D / 32 + kPage / vtb <= 32 && no_sketch && al;
}

cudaError_t launch_prefill_store_warp(const carekv_config_t& cfg, const carekv_cache_t& cache, int layer,
                                      const void* K, const void* V, int T, int seq_begin, int seq_count,
                                      const carekv_store_params_t& prm, int in_H, cudaStream_t st) {
  if (cfg.head_dim == 64) return pstore::launch_bits<64>(cfg, cache, layer, K, V, T, seq_begin, seq_count, prm, in_H, st);
  return pstore::launch_bits<128>(cfg, cache, layer, K, V, T, seq_begin, seq_count, prm, in_H, st);
}

}  // namespace carekv
