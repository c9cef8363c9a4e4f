// Fast split-K decode pass over packed INT3 pages (kernel K3, sm_100a).
//
// Same contract as decode_partial_kernel in decode.cu (logits to the
// workspace, one (m, l, O) partial per CTA), built for the HBM roofline:
//
//  * Data movement: every warp runs its own NS-stage pipeline of TMA bulk
//    copies (cp.async.bulk global->shared, completion on an mbarrier) that
//    stage CP contiguous pages at a time: packed K rows, packed V rows and
//    their int8 scale codes.  Waits are bounded; a wait that runs out sets
//    an error bit and the warp stops issuing work.
//  * Dequantization: INT3 fields are moved into fp16 mantissas with PRMT /
//    LOP3 (two's complement turned into offset binary by an XOR folded into
//    the mask), the offset is removed with HSUB2 and the group scale applied
//    with HMUL2, which rounds exactly like the reference's fp16
//    dequantization (code * scale computed exactly, rounded once to fp16).
//  * Math: Q.K_hat^T and P.V_hat run on the tensor cores (mma.sync
//    m16n8k16, fp16 inputs, fp32 accumulation).  q and p are split into
//    hi + lo fp16 halves (rows r and r+8 of the A operand) so the products
//    keep ~22 bits: the logits match an fp32 dot product to accumulation-
//    order rounding.  The channel order inside each MMA is permuted so that
//    every thread decodes whole packed words it loads itself.
//  * q . R_K of every stored K slot (for the router's combined_kvscore) on
//    the same Q rows: the slot's 4-bit codes are the B operand as exact
//    fp16 integers, the slot scale applied to the fp32 result.
#include "common.cuh"
#include "internal.h"
#include "decode_args.h"
#include "ptx.cuh"

namespace carekv {
namespace fast {

constexpr int kWarps = 4;
constexpr int kCP = 2;   // pages per stage
constexpr int kNS = 4;   // stages per warp
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t lop_and_xor(uint32_t x, uint32_t m, uint32_t k) { return (x & m) ^ k; }
__device__ __forceinline__ uint32_t dup_h2(float v) { return pack_h2(v, v); }

// 24-bit packed word w of a row (3 bytes at 3w) from two aligned 32-bit
// shared-memory loads; bits above 23 are garbage the extractors mask out.
__device__ __forceinline__ uint32_t word24(const uint8_t* row, int w) {
  const int o = 3 * w;
  const uint32_t* p = reinterpret_cast<const uint32_t*>(row + (o & ~3));
  const uint32_t lo = p[0], hi = p[1];
  return __byte_perm(lo, hi, 0x3210 + 0x1111 * (o & 3));
}

// fp16 magic for a 3-bit field placed at mantissa bit s: value 2^(10-s) + u.
// The key XORs bit 2 of the field (two's complement -> offset binary, u =
// code + 4), and the same key read as fp16 is the offset 2^(10-s) + 4.
#define CK_KEY(s) ((((25u - (s)) << 10) | (4u << (s))) * 0x00010001u)
#define CK_MASK(s) ((7u << (s)) * 0x00010001u)

// K side: the four adjacent pairs (f0,f1) (f2,f3) (f4,f5) (f6,f7) of one word,
// each as an exact fp16 half2 of code*sigma.
__device__ __forceinline__ void k_pairs(uint32_t G, uint32_t sig2, uint32_t (&o)[4]) {
  const uint32_t t = __byte_perm(G, G << 13, 0x7610);        // lo16 = G[0:16], hi16 = G[3:19]
  const uint32_t t2 = __byte_perm(G >> 12, G << 1, 0x7610);  // lo16 = G[12:28], hi16 = G[15:31]
  o[0] = h2mul(h2sub(lop_and_xor(t, CK_MASK(0), CK_KEY(0)), CK_KEY(0)), sig2);
  o[1] = h2mul(h2sub(lop_and_xor(t, CK_MASK(6), CK_KEY(6)), CK_KEY(6)), sig2);
  o[2] = h2mul(h2sub(lop_and_xor(t2, CK_MASK(0), CK_KEY(0)), CK_KEY(0)), sig2);
  o[3] = h2mul(h2sub(lop_and_xor(t2, CK_MASK(6), CK_KEY(6)), CK_KEY(6)), sig2);
}

// V side: field i of row a (low half) and of row b (high half), i = 0..7.
__device__ __forceinline__ void v_pairs(uint32_t Ga, uint32_t Gb, uint32_t sig2, uint32_t (&o)[8]) {
  const uint32_t r1 = __byte_perm(Ga, Gb, 0x5410);
  const uint32_t r2 = __byte_perm(Ga, Gb, 0x6521);
  const uint32_t r3 = __byte_perm(Ga, Gb, 0x7632);
  o[0] = h2mul(h2sub(lop_and_xor(r1, CK_MASK(0), CK_KEY(0)), CK_KEY(0)), sig2);
  o[1] = h2mul(h2sub(lop_and_xor(r1, CK_MASK(3), CK_KEY(3)), CK_KEY(3)), sig2);
  o[2] = h2mul(h2sub(lop_and_xor(r1, CK_MASK(6), CK_KEY(6)), CK_KEY(6)), sig2);
  o[3] = h2mul(h2sub(lop_and_xor(r2, CK_MASK(1), CK_KEY(1)), CK_KEY(1)), sig2);
  o[4] = h2mul(h2sub(lop_and_xor(r2, CK_MASK(4), CK_KEY(4)), CK_KEY(4)), sig2);
  o[5] = h2mul(h2sub(lop_and_xor(r2, CK_MASK(7), CK_KEY(7)), CK_KEY(7)), sig2);
  o[6] = h2mul(h2sub(lop_and_xor(r3, CK_MASK(2), CK_KEY(2)), CK_KEY(2)), sig2);
  o[7] = h2mul(h2sub(lop_and_xor(r3, CK_MASK(5), CK_KEY(5)), CK_KEY(5)), sig2);
}

template <int D>
struct StageLayout {
  static constexpr int R = D * 3 / 8;
  static constexpr int G = D / 32;       // int8 scale bytes per row at group 32 (max)
  static constexpr int kBytes = kCP * kPage * R;
  static constexpr int kPad = 16;
  static constexpr int sBytesMax = kCP * kPage * 4;  // scale bytes (G <= 4)
  static constexpr int kOff = 0;
  static constexpr int vOff = kBytes + kPad;
  static constexpr int ksOff = vOff + kBytes + kPad;
  static constexpr int vsOff = ksOff + sBytesMax;
  static constexpr int bytes = ((vsOff + sBytesMax + 127) / 128) * 128;
};

// One warp's state.  QN query heads share the kv head (<= 8).
template <int QN, int D>
__global__ void __launch_bounds__(kWarps * 32, 2) decode_partial_int3(DecodeArgs a) {
  using SL = StageLayout<D>;
  constexpr int KSTEPS = D / 16;  // k-steps of Q.K^T
  constexpr int NT = D / 8;       // n-tiles of P.V
  constexpr int KW = D / 32;      // packed words per thread on the K side
  constexpr int VW = D / 64;      // packed words per thread on the V side (D=64 -> 1)
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bars[kWarps][kNS];
  __shared__ float sm_m[kWarps][8], sm_l[kWarps][8];
  // A fragments of the slot dots per 32-channel group and k-step: rows gid =
  // q_hi, gid+8 = q_lo of query gid; k-step ks covers channels
  // 8*tig + 4*ks + {0..3} of the group (the nibble order of a payload word)
  __shared__ __align__(16) uint32_t qfr[D / 32][2][32][4];

  const Dims d = make_dims(a.cfg);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  const int bh = blockIdx.x, split = blockIdx.y;
  const int s = bh / d.H, h = bh % d.H, b = a.seq_begin + s;
  const int64_t lhp = d.lhp(b, a.layer, h);
  const int np = min(a.cache.num_pages[lhp], a.p_used);
  const int ca = split * a.pps, cb = min(np, ca + a.pps);
  const int n_cta = max(0, cb - ca);
  const int qv = n_cta / kWarps, rv = n_cta % kWarps;
  const int pa = ca + warp * qv + min(warp, rv);
  const int pb = pa + qv + (warp < rv ? 1 : 0);
  const int G = d.G;                 // scale bytes per row
  const int gsz = d.gsize;
  const int Hq = a.act_heads;   // query heads per activation row

  uint8_t* wsm = smem + warp * (kNS * SL::bytes);
  uint64_t* bar = bars[warp];
  if (lane == 0) {
    for (int i = 0; i < kNS; ++i) mbar_init(&bar[i], 1);
    fence_mbar_init();
  }
  __syncwarp();

  // ── A fragments of Q (hi rows gid, lo rows gid+8), channel-permuted ──
  uint32_t qa[KSTEPS][4];
  {
    const int c0 = tig * (D / 4);
#pragma unroll
    for (int kb = 0; kb < KSTEPS; ++kb) {
      float q4[4] = {0.f, 0.f, 0.f, 0.f};
      if (gid < QN) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          q4[j] = load_act(a.q, (static_cast<int64_t>(s) * Hq + h * QN + gid) * D + c0 + 4 * kb + j, a.dt);
      }
      float hi[4], lo[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        hi[j] = __half2float(__float2half_rn(q4[j]));
        lo[j] = q4[j] - hi[j];
      }
      qa[kb][0] = pack_h2(hi[0], hi[1]);
      qa[kb][1] = pack_h2(lo[0], lo[1]);
      qa[kb][2] = pack_h2(hi[2], hi[3]);
      qa[kb][3] = pack_h2(lo[2], lo[3]);
    }
  }

  float o[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_run = -INFINITY, l_part = 0.f;
  float* Srow = a.S + (static_cast<int64_t>(bh) * QN + gid) * a.p_used * kPage;
  const bool kslot = a.kw != nullptr;
  if (kslot) {
    for (int x = threadIdx.x; x < (D / 32) * 2 * 32; x += blockDim.x) {
      const int g = x / 64, ks = (x / 32) % 2, ln = x % 32;
      const int qg = ln >> 2, tg = ln & 3;
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      if (qg < QN)
#pragma unroll
        for (int e = 0; e < 4; ++e)
          v[e] = load_act(a.q, (static_cast<int64_t>(s) * Hq + h * QN + qg) * D + g * 32 + 8 * tg + 4 * ks + e, a.dt);
      float hi[4], lo[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        hi[e] = __half2float(__float2half_rn(v[e]));
        lo[e] = v[e] - hi[e];
      }
      qfr[g][ks][ln][0] = pack_h2(hi[0], hi[1]);
      qfr[g][ks][ln][1] = pack_h2(lo[0], lo[1]);
      qfr[g][ks][ln][2] = pack_h2(hi[2], hi[3]);
      qfr[g][ks][ln][3] = pack_h2(lo[2], lo[3]);
    }
    __syncthreads();
  }
  const int KG = a.p_used * d.SK;
  float* Wrow = kslot ? a.kw + (static_cast<int64_t>(bh) * QN + gid) * KG * kPage : nullptr;

  const int n_chunks = (pb - pa + kCP - 1) / kCP;
  const int64_t page0 = lhp * d.P;
  auto issue = [&](int c) {
    const int p = pa + c * kCP;
    const int n = min(kCP, pb - p);
    uint8_t* st = wsm + (c % kNS) * SL::bytes;
    const uint32_t cb_ = n * kPage * d.R, sb = n * kPage * G;
    mbar_expect_tx(&bar[c % kNS], 2 * cb_ + 2 * sb);
    bulk_g2s(st + SL::kOff, a.cache.k_codes + (page0 + p) * kPage * d.R, cb_, &bar[c % kNS]);
    bulk_g2s(st + SL::vOff, a.cache.v_codes + (page0 + p) * kPage * d.R, cb_, &bar[c % kNS]);
    bulk_g2s(st + SL::ksOff, reinterpret_cast<const int8_t*>(a.cache.k_scale) + (page0 + p) * kPage * G, sb,
             &bar[c % kNS]);
    bulk_g2s(st + SL::vsOff, reinterpret_cast<const int8_t*>(a.cache.v_scale) + (page0 + p) * kPage * G, sb,
             &bar[c % kNS]);
  };
  if (lane == 0)
    for (int c = 0; c < min(kNS, n_chunks); ++c) issue(c);

  bool failed = false;
  int fail_chunk = n_chunks;
  for (int c = 0; c < n_chunks && !failed; ++c) {
    if (!mbar_wait(&bar[c % kNS], (c / kNS) & 1)) {
      failed = true;
      fail_chunk = c;
      if (lane == 0) atomicOr(a.cache.error_flag, 4);
      break;
    }
    const uint8_t* st = wsm + (c % kNS) * SL::bytes;
    const int pbase = pa + c * kCP;
    const int npg = min(kCP, pb - pbase);
    for (int pp = 0; pp < npg; ++pp) {
      const int p = pbase + pp;
      const int64_t pg = page0 + p;
      const int nv = a.cache.valid[pg];
      const float mk = f16_bits_to_f32(a.cache.k_master[pg]);
      const float mv = f16_bits_to_f32(a.cache.v_master[pg]);
      const uint8_t* kc = st + SL::kOff + pp * kPage * d.R;
      const uint8_t* vc = st + SL::vOff + pp * kPage * d.R;
      const int8_t* ks = reinterpret_cast<const int8_t*>(st + SL::ksOff) + pp * kPage * G;
      const int8_t* vs = reinterpret_cast<const int8_t*>(st + SL::vsOff) + pp * kPage * G;

      // ── logits: S = Q_hl . K_hat^T, two n-tiles of 8 tokens ──
      float sv[2][2];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int row = nt * 8 + gid;
        const uint8_t* kr = kc + row * d.R;
        const int gk = (tig * (D / 4)) / gsz;
        const float sig = f16r(__fmul_rn(static_cast<float>(ks[row * G + gk]), mk));
        const uint32_t sig2 = dup_h2(sig);
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int w = 0; w < KW; ++w) {
          uint32_t kp[4];
          k_pairs(word24(kr, tig * KW + w), sig2, kp);
          mma16816(acc, qa[2 * w], kp[0], kp[1]);
          mma16816(acc, qa[2 * w + 1], kp[2], kp[3]);
        }
        sv[nt][0] = __fmul_rn(acc[0] + acc[2], a.sf);
        sv[nt][1] = __fmul_rn(acc[1] + acc[3], a.sf);
      }
      // store logits of valid tokens (rows gid < QN)
      if (gid < QN) {
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const int t = nt * 8 + 2 * tig;
          if (t + 1 < nv) {
            *reinterpret_cast<float2*>(Srow + p * kPage + t) = make_float2(sv[nt][0], sv[nt][1]);
          } else if (t < nv) {
            Srow[p * kPage + t] = sv[nt][0];
          }
        }
      }
      // ── q . R_K of the page's stored K slots: tokens 2tig, 2tig+1 (c0)
      // and 8+2tig, 9+2tig (c1) of query gid, times the slot scale ──
      if (kslot && nv > 0) {
        for (int j = 0; j < d.SK; ++j) {
          const int grp = a.cache.k_slot_group[pg * d.SK + j];
          if (grp < 0 || grp >= D / 32) continue;
          const uint8_t* pay = a.cache.k_slot_data + (pg * d.SK + j) * d.kslot_bytes;
          const uint32_t w0 = *reinterpret_cast<const uint32_t*>(pay + gid * 16 + 4 * tig);
          const uint32_t w1 = *reinterpret_cast<const uint32_t*>(pay + (gid + 8) * 16 + 4 * tig);
          const float rs = f16_bits_to_f32(a.cache.k_slot_scale[pg * d.SK + j]);
          float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int ks = 0; ks < 2; ++ks) {
            const uint4 af = *reinterpret_cast<const uint4*>(&qfr[grp][ks][lane][0]);
            mma_f16(c0, af.x, af.y, af.z, af.w, nib_pair(w0, 2 * ks), nib_pair(w0, 2 * ks + 1));
            mma_f16(c1, af.x, af.y, af.z, af.w, nib_pair(w1, 2 * ks), nib_pair(w1, 2 * ks + 1));
          }
          if (gid < QN) {
            float* wr = Wrow + (static_cast<int64_t>(p) * d.SK + j) * kPage;
            *reinterpret_cast<float2*>(wr + 2 * tig) =
                make_float2(__fmul_rn(c0[0] + c0[2], rs), __fmul_rn(c0[1] + c0[3], rs));
            *reinterpret_cast<float2*>(wr + 8 + 2 * tig) =
                make_float2(__fmul_rn(c1[0] + c1[2], rs), __fmul_rn(c1[1] + c1[3], rs));
          }
        }
      }
      // ── online softmax (per query row gid; the quad holds 16 tokens) ──
      float pmax = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e)
          if (nt * 8 + 2 * tig + e < nv) pmax = fmaxf(pmax, sv[nt][e]);
      pmax = fmaxf(pmax, __shfl_xor_sync(0xffffffffu, pmax, 1));
      pmax = fmaxf(pmax, __shfl_xor_sync(0xffffffffu, pmax, 2));
      const float m_new = fmaxf(m_run, pmax);
      if (m_new > m_run) {
        const float alpha = m_run == -INFINITY ? 0.f : exp2f((m_run - m_new) * kLog2e);
        l_part *= alpha;
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          o[j][0] *= alpha; o[j][1] *= alpha; o[j][2] *= alpha; o[j][3] *= alpha;
        }
        m_run = m_new;
      }
      float pr[2][2];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float x = (nt * 8 + 2 * tig + e < nv) ? exp2f((sv[nt][e] - m_run) * kLog2e) : 0.f;
          pr[nt][e] = x;
          l_part += x;
        }
      uint32_t pa_[4];
      {
        const float h00 = __half2float(__float2half_rn(pr[0][0])), h01 = __half2float(__float2half_rn(pr[0][1]));
        const float h10 = __half2float(__float2half_rn(pr[1][0])), h11 = __half2float(__float2half_rn(pr[1][1]));
        pa_[0] = pack_h2(h00, h01);
        pa_[1] = pack_h2(pr[0][0] - h00, pr[0][1] - h01);
        pa_[2] = pack_h2(h10, h11);
        pa_[3] = pack_h2(pr[1][0] - h10, pr[1][1] - h11);
      }
      // ── O += P . V_hat: rows (2tig, 2tig+1) and (2tig+8, 2tig+9) ──
      const int gv = (gid * (D / 8)) / gsz;
      const int r0 = 2 * tig, r1 = 2 * tig + 8;
      const uint32_t siga = pack_h2(f16r(__fmul_rn(static_cast<float>(vs[r0 * G + gv]), mv)),
                                    f16r(__fmul_rn(static_cast<float>(vs[(r0 + 1) * G + gv]), mv)));
      const uint32_t sigb = pack_h2(f16r(__fmul_rn(static_cast<float>(vs[r1 * G + gv]), mv)),
                                    f16r(__fmul_rn(static_cast<float>(vs[(r1 + 1) * G + gv]), mv)));
#pragma unroll
      for (int w = 0; w < (VW > 0 ? VW : 1); ++w) {
        const int wi = gid * (VW > 0 ? VW : 1) + w;
        uint32_t va[8], vb[8];
        v_pairs(word24(vc + r0 * d.R, wi), word24(vc + (r0 + 1) * d.R, wi), siga, va);
        v_pairs(word24(vc + r1 * d.R, wi), word24(vc + (r1 + 1) * d.R, wi), sigb, vb);
#pragma unroll
        for (int f = 0; f < 8; ++f) mma16816(o[w * 8 + f], pa_, va[f], vb[f]);
      }
    }
    __syncwarp();
    if (lane == 0 && c + kNS < n_chunks) {
      fence_proxy_async();
      issue(c + kNS);
    }
  }
  if (failed && lane == 0) {
    // let the copies already issued land (bounded) before the staging area
    // is reused or the CTA exits
    for (int c2 = 0; c2 < n_chunks; ++c2) {
      if (c2 < fail_chunk || c2 >= fail_chunk + kNS) continue;
      (void)mbar_wait(&bar[c2 % kNS], (c2 / kNS) & 1);
    }
  }

  // ── merge: per query row gid, quad-reduce l, then the 4 warps ──
  l_part += __shfl_xor_sync(0xffffffffu, l_part, 1);
  l_part += __shfl_xor_sync(0xffffffffu, l_part, 2);
  float* so = reinterpret_cast<float*>(smem);  // reuse the staging area (all warps are past it)
  __syncthreads();
  if (tig == 0) {
    sm_m[warp][gid] = m_run;
    sm_l[warp][gid] = l_part;
  }
  // O rows: hi (c0,c1) + lo (c2,c3) for query gid, channels of n-tile j
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int c0 = (2 * tig) * (D / 8) + j;
    const int c1 = (2 * tig + 1) * (D / 8) + j;
    so[(warp * 8 + gid) * D + c0] = o[j][0] + o[j][2];
    so[(warp * 8 + gid) * D + c1] = o[j][1] + o[j][3];
  }
  __syncthreads();
  const int64_t part = static_cast<int64_t>(bh) * a.n_splits + split;
  for (int idx = threadIdx.x; idx < QN * D; idx += blockDim.x) {
    const int i = idx / D, cidx = idx % D;
    float M = -INFINITY;
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, sm_m[w][i]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
      for (int w = 0; w < kWarps; ++w) {
        if (sm_m[w][i] == -INFINITY) continue;
        const float f = exp2f((sm_m[w][i] - M) * kLog2e);
        L += sm_l[w][i] * f;
        O += so[(w * 8 + i) * D + cidx] * f;
      }
    }
    a.po[(part * QN + i) * D + cidx] = O;
    if (cidx == 0) {
      a.pm[part * QN + i] = M;
      a.pl[part * QN + i] = L;
    }
  }
}

}  // namespace fast

template <int QN, int D>
cudaError_t launch_decode_partial_int3(DecodeArgs& a, cudaStream_t st, int n_bh) {
  constexpr int smem = fast::kWarps * fast::kNS * fast::StageLayout<D>::bytes;
  static bool attr_set = false;  // per process; the attribute is per function, not per device
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(fast::decode_partial_int3<QN, D>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  dim3 grid(n_bh, a.n_splits);
  fast::decode_partial_int3<QN, D><<<grid, fast::kWarps * 32, smem, st>>>(a);
  return cudaGetLastError();
}

#define CK_INST(QN, D) template cudaError_t launch_decode_partial_int3<QN, D>(DecodeArgs&, cudaStream_t, int);
CK_INST(1, 64) CK_INST(2, 64) CK_INST(4, 64) CK_INST(8, 64)
CK_INST(1, 128) CK_INST(2, 128) CK_INST(4, 128) CK_INST(8, 128)
#undef CK_INST

}  // namespace carekv
