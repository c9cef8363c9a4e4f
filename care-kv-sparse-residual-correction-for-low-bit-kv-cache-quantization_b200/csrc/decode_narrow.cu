// Narrow-group split-K decode pass over packed INT3 pages (kernel K3n,
// sm_100a): kv heads whose query group has at most 4 heads (MHA, GQA-2,
// GQA-4).
//
// Contract: like the wide pass in decode_fast.cu, every CTA streams a range
// of pages of one (sequence, kv head) and writes the logits S of every token
// and one (m, l, O) split partial.  In addition, when live combined_kvscore
// scoring is on (attention.py:167-184), it writes w = q . R_K for every
// stored K residual slot, query and token (R_K = code * slot scale over the
// slot's 32-channel group), so the router never re-reads slot payloads.
//
// Orientation: tokens and channels sit on the M side of the MMAs and the
// queries on N, as 8 columns = fp16 hi and lo halves of up to 4 queries:
//     S^T [16 tok x 8]  = K_hat [16 tok x D] . Q^T [D x 8]
//     O^T [D x 8]      += V_hat^T [D x 16 tok] . P^T [16 tok x 8]
//     w^T [16 tok x 8]  = R_K [16 tok x 32] . Q_g^T [32 x 8]
// A page costs D/16 MMAs per side, each thread keeps D/4 fp32 accumulators,
// and the hi + lo split keeps ~22 significant bits of q and p, so S and O
// match an fp32 evaluation to accumulation-order rounding.
//
// Per warp: an NS-stage ring of bulk copies (cp.async.bulk + mbarrier,
// bounded waits) stages CP contiguous pages at a time: packed K and V rows,
// their int8 scale codes and the pages' K slot payloads.  Per-page metadata
// (valid rows, fp16 masters, slot groups and scales) is read 32 pages at a
// time into shared memory.  Dequantization is exact: 3-bit fields are moved
// into fp16 mantissas (PRMT / LOP3), the offset removed with HSUB2 and the
// scale applied with HMUL2, i.e. fp16(code * scale) rounded once, as the
// reference dequantizes; scale codes become fp16(int8 * master) the same way.
#include "common.cuh"
#include "internal.h"
#include "decode_args.h"
#include "ptx.cuh"

namespace carekv {
namespace narrow {

constexpr int kWarps = 4;
constexpr int kCP = 2;    // pages per stage
constexpr int kNS = 3;    // stages per warp
constexpr int kWin = 32;  // pages per metadata window
constexpr float kLog2e = 1.4426950408889634f;

// Stage geometry (bytes); the 16-byte pads after the code blocks absorb the
// aligned 8-byte reads of a row's last packed word.
struct Geo {
  int R, G, SK, kbytes, vOff, ksOff, vsOff, slOff, stage, meta, qs, total;
};
__host__ __device__ inline Geo geo(int D, int G, int SK, bool kslot) {
  Geo g;
  g.R = D * 3 / 8;
  g.G = G;
  g.SK = SK;
  g.kbytes = kCP * kPage * g.R;
  g.vOff = g.kbytes + 16;
  g.ksOff = g.vOff + g.kbytes + 16;
  g.vsOff = g.ksOff + kCP * kPage * G;
  g.slOff = g.vsOff + kCP * kPage * G;
  g.stage = (g.slOff + (kslot ? kCP * SK * 256 : 0) + 127) & ~127;
  // per warp: valid, km2, vm2 per page, then (group, scale) per page and slot
  g.meta = kWin * 12 + (kslot ? kWin * SK * 8 : 0);
  g.qs = kslot ? (D / 32) * 2 * 32 * 8 : 0;
  g.total = kWarps * kNS * g.stage + kWarps * g.meta + g.qs;
  return g;
}

__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }

// 24-bit packed word at byte offset o of a staged row (bits 24..31 garbage).
__device__ __forceinline__ uint32_t word24_at(const uint8_t* row, int o) {
  const uint32_t* p = reinterpret_cast<const uint32_t*>(row + (o & ~3));
  return prmt(p[0], p[1], 0x3210 + 0x1111 * (o & 3));
}

// One packed word (8 codes f0..f7, 3 bits each) of a K row -> the four half2
// operands of two k-steps: (f0,f3) (f1,f4) | (f2,f5) (f6,f7).
__device__ __forceinline__ void k_quads(uint32_t W, uint32_t sig2, uint32_t (&o)[4]) {
  const uint32_t t1 = prmt(W, W, 0x2110);  // low half W[0:16], high half W[8:24]
  const uint32_t t2 = prmt(W, W, 0x2222);  // both halves W[16:24] in their low byte
  o[0] = i3_pair<0, 1>(t1, sig2);
  o[1] = i3_pair<3, 4>(t1, sig2);
  o[2] = i3_pair<6, 7>(t1, sig2);
  o[3] = i3_pair<2, 5>(t2, sig2);
}
// Same word of rows a (low half) and b (high half): field f of both rows.
__device__ __forceinline__ void v_octs(uint32_t Wa, uint32_t Wb, uint32_t sig2, uint32_t (&o)[8]) {
  const uint32_t r1 = prmt(Wa, Wb, 0x5410);
  const uint32_t r2 = prmt(Wa, Wb, 0x6521);
  const uint32_t r3 = prmt(Wa, Wb, 0x7632);
  o[0] = i3_pair<0, 0>(r1, sig2);
  o[1] = i3_pair<3, 3>(r1, sig2);
  o[2] = i3_pair<6, 6>(r1, sig2);
  o[3] = i3_pair<1, 1>(r2, sig2);
  o[4] = i3_pair<4, 4>(r2, sig2);
  o[5] = i3_pair<7, 7>(r2, sig2);
  o[6] = i3_pair<2, 2>(r3, sig2);
  o[7] = i3_pair<5, 5>(r3, sig2);
}

// fp16 hi / lo halves of x packed as (hi, lo)
__device__ __forceinline__ uint32_t hilo(float x) {
  const __half hi = __float2half_rn(x);
  const __half lo = __float2half_rn(x - __half2float(hi));
  __half2 r = __halves2half2(hi, lo);
  return *reinterpret_cast<uint32_t*>(&r);
}

template <int QN, int D>
__global__ void __launch_bounds__(kWarps * 32, 4) decode_narrow(DecodeArgs a) {
  constexpr int R = D * 3 / 8;
  constexpr int KS = D / 16;   // k-steps of Q.K^T = m-tiles of O^T
  constexpr int KW = D / 32;   // packed K words per thread and row
  constexpr int G4 = D / 32;   // 32-channel groups (K residual slots)
  static_assert(QN >= 1 && QN <= 4, "narrow pass: at most 4 queries per kv head");
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bars[kWarps][kNS];
  __shared__ float sm_m[kWarps][4], sm_l[kWarps][4];

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
  const int Hq = d.H * QN;
  const int G = d.G, SK = d.SK;
  const bool kslot = a.kw != nullptr;
  const Geo g = geo(D, G, SK, kslot);
  const int64_t page0 = lhp * d.P;
  const int KG = a.p_used * SK;

  uint8_t* wsm = smem + warp * (kNS * g.stage);
  uint8_t* meta = smem + kWarps * kNS * g.stage + warp * g.meta;
  int* m_valid = reinterpret_cast<int*>(meta);
  uint32_t* m_km = reinterpret_cast<uint32_t*>(meta + kWin * 4);
  uint32_t* m_vm = reinterpret_cast<uint32_t*>(meta + kWin * 8);
  int* m_grp = reinterpret_cast<int*>(meta + kWin * 12);
  float* m_rs = reinterpret_cast<float*>(meta + kWin * 12 + kWin * SK * 4);
  uint2* qs = reinterpret_cast<uint2*>(smem + kWarps * kNS * g.stage + kWarps * g.meta);
  uint64_t* bar = bars[warp];

  if (lane == 0) {
    for (int i = 0; i < kNS; ++i) mbar_init(&bar[i], 1);
    fence_mbar_init();
  }
  __syncwarp();

  const int n_chunks = (pb - pa + kCP - 1) / kCP;
  auto issue = [&](int c) {
    const int p = pa + c * kCP;
    const int n = min(kCP, pb - p);
    uint8_t* st = wsm + (c % kNS) * g.stage;
    uint64_t* br = &bar[c % kNS];
    const uint32_t cbytes = n * kPage * R, sbytes = n * kPage * G;
    const uint32_t slbytes = kslot ? n * SK * 256 : 0;
    mbar_expect_tx(br, 2 * cbytes + 2 * sbytes + slbytes);
    bulk_g2s(st, a.cache.k_codes + (page0 + p) * kPage * R, cbytes, br);
    bulk_g2s(st + g.vOff, a.cache.v_codes + (page0 + p) * kPage * R, cbytes, br);
    bulk_g2s(st + g.ksOff, reinterpret_cast<const int8_t*>(a.cache.k_scale) + (page0 + p) * kPage * G, sbytes, br);
    bulk_g2s(st + g.vsOff, reinterpret_cast<const int8_t*>(a.cache.v_scale) + (page0 + p) * kPage * G, sbytes, br);
    if (slbytes) bulk_g2s(st + g.slOff, a.cache.k_slot_data + (page0 + p) * SK * 256, slbytes, br);
  };
  if (lane == 0)
    for (int c = 0; c < min(kNS, n_chunks); ++c) issue(c);

  // ── Q^T operands: column n = query n/2, half n%2 (0 = hi, 1 = lo) ──
  const int qi = gid >> 1, part = gid & 1;
  auto qval = [&](int c) -> float {
    if (qi >= QN) return 0.f;
    const float x = load_act(a.q, (static_cast<int64_t>(s) * Hq + h * QN + qi) * D + c, a.dt);
    const float hi = __half2float(__float2half_rn(x));
    return part ? x - hi : hi;
  };
  // K side: thread tig owns channels tig*D/4 .. +D/4 (KW packed words); word
  // i feeds k-steps 2i ((f0,f3) (f1,f4)) and 2i+1 ((f2,f5) (f6,f7)).
  uint32_t qb[KS][2];
  {
    const int c0 = tig * (D / 4);
#pragma unroll
    for (int i = 0; i < KW; ++i) {
      const int c = c0 + 8 * i;
      qb[2 * i][0] = pack_h2(qval(c + 0), qval(c + 3));
      qb[2 * i][1] = pack_h2(qval(c + 1), qval(c + 4));
      qb[2 * i + 1][0] = pack_h2(qval(c + 2), qval(c + 5));
      qb[2 * i + 1][1] = pack_h2(qval(c + 6), qval(c + 7));
    }
  }
  // slot operands per 32-channel group: k-step ks takes channels
  // 8*tig + 4*ks + {0,1} and {2,3} of the group (one nibble word per token)
  if (kslot) {
    for (int x = threadIdx.x; x < G4 * 2 * 32; x += blockDim.x) {
      const int grp = x / 64, ks = (x / 32) % 2, ln = x % 32;
      const int lq = (ln >> 2) >> 1, lp = (ln >> 2) & 1, lt = ln & 3;
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      if (lq < QN)
        for (int e = 0; e < 4; ++e) {
          const float xq = load_act(a.q, (static_cast<int64_t>(s) * Hq + h * QN + lq) * D + grp * 32 + 8 * lt +
                                             4 * ks + e, a.dt);
          const float hi = __half2float(__float2half_rn(xq));
          v[e] = lp ? xq - hi : hi;
        }
      qs[x] = make_uint2(pack_h2(v[0], v[1]), pack_h2(v[2], v[3]));
    }
    __syncthreads();
  }

  float o[KS][4];
#pragma unroll
  for (int j = 0; j < KS; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_run = -INFINITY, l_part = 0.f;
  float* Srow = a.S + (static_cast<int64_t>(bh) * QN + tig) * a.p_used * kPage;
  float* Wrow = kslot ? a.kw + (static_cast<int64_t>(bh) * QN + tig) * KG * kPage : nullptr;
  const bool q_ok = tig < QN;

  // V side: thread gid owns packed words (D=128) 2gid, 2gid+1 / (D=64) gid
  constexpr int VB = D == 128 ? 6 : 3;  // byte offset multiplier of the thread's first word
  const int vo = VB * gid;
  const int vbase = vo & ~3, voff = vo & 3;
  const uint32_t vsel_l = 0x3210 + 0x1111 * voff;
  const uint32_t vsel_h = (0x3210 + 0x1111 * (voff + 3)) & 0x7777;
  const int gk = (tig * (D / 4)) / d.gsize;            // K scale group of the thread's channels
  const int gv = ((D == 128 ? 16 : 8) * gid) / d.gsize;  // V scale group
  const int ra = 2 * tig;                               // V rows ra, ra+1, ra+8, ra+9
  const uint32_t psel = part ? 0x7632u : 0x5410u;
  const int src_a = 8 * tig + qi, src_b = src_a + 4;

  bool failed = false;
  int fail_chunk = n_chunks;
  for (int c = 0; c < n_chunks; ++c) {
    const int pbase = pa + c * kCP;
    if (((pbase - pa) % kWin) == 0) {
      // per-page metadata of the next window
      __syncwarp();
      const int p = pbase + lane;
      int nv = 0;
      uint32_t km = 0, vm = 0;
      if (p < pb) {
        nv = a.cache.valid[page0 + p];
        km = a.cache.k_master[page0 + p];
        vm = a.cache.v_master[page0 + p];
      }
      m_valid[lane] = nv;
      m_km[lane] = km | (km << 16);
      m_vm[lane] = vm | (vm << 16);
      if (kslot) {
        for (int j = 0; j < SK; ++j) {
          int grp = -1;
          float rs = 0.f;
          if (p < pb) {
            grp = a.cache.k_slot_group[(page0 + p) * SK + j];
            rs = f16_bits_to_f32(a.cache.k_slot_scale[(page0 + p) * SK + j]);
          }
          m_grp[lane * SK + j] = grp;
          m_rs[lane * SK + j] = rs;
        }
      }
      __syncwarp();
    }
    if (!mbar_wait(&bar[c % kNS], (c / kNS) & 1)) {
      failed = true;
      fail_chunk = c;
      if (lane == 0) atomicOr(a.cache.error_flag, 4);
      break;
    }
    const uint8_t* st = wsm + (c % kNS) * g.stage;
    const int npg = min(kCP, pb - pbase);
    for (int pp = 0; pp < npg; ++pp) {
      const int p = pbase + pp;
      const int mi = (p - pa) % kWin;
      const int nv = m_valid[mi];
      const uint32_t km2 = m_km[mi], vm2 = m_vm[mi];
      const uint8_t* kc = st + pp * kPage * R;
      const uint8_t* vc = st + g.vOff + pp * kPage * R;
      const uint8_t* ks = st + g.ksOff + pp * kPage * G;
      const uint8_t* vs = st + g.vsOff + pp * kPage * G;

      // ── S^T = K_hat . Q^T: rows gid, gid+8 ──
      float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      {
        const uint32_t sig = i8_scale_pair(static_cast<uint32_t>(ks[gid * G + gk]) |
                                               (static_cast<uint32_t>(ks[(gid + 8) * G + gk]) << 16),
                                           km2);
        const uint32_t sig0 = prmt(sig, sig, 0x1010), sig8 = prmt(sig, sig, 0x3232);
        uint32_t w0[KW], w8[KW];
        if constexpr (D == 128) {
          const uint8_t* r0 = kc + gid * R + 12 * tig;
          const uint8_t* r8 = r0 + 8 * R;
          const uint32_t x0 = lds32(r0), x1 = lds32(r0 + 4), x2 = lds32(r0 + 8);
          const uint32_t y0 = lds32(r8), y1 = lds32(r8 + 4), y2 = lds32(r8 + 8);
          w0[0] = x0; w0[1] = prmt(x0, x1, 0x6543); w0[2] = prmt(x1, x2, 0x5432); w0[3] = x2 >> 8;
          w8[0] = y0; w8[1] = prmt(y0, y1, 0x6543); w8[2] = prmt(y1, y2, 0x5432); w8[3] = y2 >> 8;
        } else {
#pragma unroll
          for (int i = 0; i < KW; ++i) {
            w0[i] = word24_at(kc + gid * R, 6 * tig + 3 * i);
            w8[i] = word24_at(kc + (gid + 8) * R, 6 * tig + 3 * i);
          }
        }
#pragma unroll
        for (int i = 0; i < KW; ++i) {
          uint32_t p0[4], p8[4];
          k_quads(w0[i], sig0, p0);
          k_quads(w8[i], sig8, p8);
          mma_f16(acc[i & 1], p0[0], p8[0], p0[1], p8[1], qb[2 * i][0], qb[2 * i][1]);
          mma_f16(acc[i & 1], p0[2], p8[2], p0[3], p8[3], qb[2 * i + 1][0], qb[2 * i + 1][1]);
        }
      }
      const float s0 = __fmul_rn((acc[0][0] + acc[1][0]) + (acc[0][1] + acc[1][1]), a.sf);
      const float s1 = __fmul_rn((acc[0][2] + acc[1][2]) + (acc[0][3] + acc[1][3]), a.sf);
      const bool t0 = gid < nv, t1 = gid + 8 < nv;
      if (q_ok) {
        Srow[p * kPage + gid] = s0;
        Srow[p * kPage + gid + 8] = s1;
      }

      // ── w = q . R_K of the page's stored K slots ──
      if (kslot) {
        const int mrow = mi * SK;
        for (int j = 0; j < SK; ++j) {
          const int grp = m_grp[mrow + j];
          if (grp < 0 || grp >= G4 || nv == 0) continue;
          const uint8_t* sl = st + g.slOff + (pp * SK + j) * 256;
          const uint32_t u0 = lds32(sl + gid * 16 + 4 * tig);
          const uint32_t u8 = lds32(sl + (gid + 8) * 16 + 4 * tig);
          const uint2 b0 = qs[(grp * 2 + 0) * 32 + lane];
          const uint2 b1 = qs[(grp * 2 + 1) * 32 + lane];
          float cw[4] = {0.f, 0.f, 0.f, 0.f};
          mma_f16(cw, nib_pair(u0, 0), nib_pair(u8, 0), nib_pair(u0, 1), nib_pair(u8, 1), b0.x, b0.y);
          mma_f16(cw, nib_pair(u0, 2), nib_pair(u8, 2), nib_pair(u0, 3), nib_pair(u8, 3), b1.x, b1.y);
          const float rs = m_rs[mrow + j];
          if (q_ok) {
            float* wr = Wrow + (static_cast<int64_t>(p) * SK + j) * kPage;
            wr[gid] = __fmul_rn(cw[0] + cw[1], rs);
            wr[gid + 8] = __fmul_rn(cw[2] + cw[3], rs);
          }
        }
      }

      // ── online softmax for query tig over the page's 16 tokens ──
      float pmax = fmaxf(t0 ? s0 : -INFINITY, t1 ? s1 : -INFINITY);
      pmax = fmaxf(pmax, __shfl_xor_sync(0xffffffffu, pmax, 4));
      pmax = fmaxf(pmax, __shfl_xor_sync(0xffffffffu, pmax, 8));
      pmax = fmaxf(pmax, __shfl_xor_sync(0xffffffffu, pmax, 16));
      const float m_new = fmaxf(m_run, pmax);
      if (__any_sync(0xffffffffu, m_new > m_run)) {
        const float alpha = m_new > m_run ? (m_run == -INFINITY ? 0.f : exp2f((m_run - m_new) * kLog2e)) : 1.f;
        l_part *= alpha;
#pragma unroll
        for (int j = 0; j < KS; ++j) {
          o[j][0] *= alpha; o[j][1] *= alpha; o[j][2] *= alpha; o[j][3] *= alpha;
        }
        m_run = m_new;
      }
      const float pr0 = t0 ? exp2f((s0 - m_run) * kLog2e) : 0.f;
      const float pr1 = t1 ? exp2f((s1 - m_run) * kLog2e) : 0.f;
      l_part += pr0 + pr1;
      // P^T operand: tokens 2tig, 2tig+1 | 2tig+8, 2tig+9 of query qi
      const uint32_t h0 = hilo(pr0), h1 = hilo(pr1);
      const uint32_t xa = __shfl_sync(0xffffffffu, h0, src_a), xb = __shfl_sync(0xffffffffu, h0, src_b);
      const uint32_t ya = __shfl_sync(0xffffffffu, h1, src_a), yb = __shfl_sync(0xffffffffu, h1, src_b);
      const uint32_t pb0 = prmt(xa, xb, psel), pb1 = prmt(ya, yb, psel);

      // ── O^T += V_hat^T . P^T ──
      const uint32_t sA = i8_scale_pair(static_cast<uint32_t>(vs[ra * G + gv]) |
                                            (static_cast<uint32_t>(vs[(ra + 1) * G + gv]) << 16),
                                        vm2);
      const uint32_t sB = i8_scale_pair(static_cast<uint32_t>(vs[(ra + 8) * G + gv]) |
                                            (static_cast<uint32_t>(vs[(ra + 9) * G + gv]) << 16),
                                        vm2);
      if constexpr (D == 128) {
        uint32_t wl[4], wh[4];
        const int rows[4] = {ra, ra + 1, ra + 8, ra + 9};
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const uint8_t* rp = vc + rows[r] * R + vbase;
          const uint32_t lo = lds32(rp), hi = lds32(rp + 4);
          wl[r] = prmt(lo, hi, vsel_l);
          wh[r] = prmt(lo, hi, vsel_h);
        }
        uint32_t al[8], ah[8], bl[8], bhh[8];
        v_octs(wl[0], wl[1], sA, al);
        v_octs(wh[0], wh[1], sA, ah);
        v_octs(wl[2], wl[3], sB, bl);
        v_octs(wh[2], wh[3], sB, bhh);
#pragma unroll
        for (int f = 0; f < 8; ++f) mma_f16(o[f], al[f], ah[f], bl[f], bhh[f], pb0, pb1);
      } else {
        uint32_t wv[4];
        const int rows[4] = {ra, ra + 1, ra + 8, ra + 9};
#pragma unroll
        for (int r = 0; r < 4; ++r) wv[r] = word24_at(vc + rows[r] * R, vo);
        uint32_t va[8], vb[8];
        v_octs(wv[0], wv[1], sA, va);
        v_octs(wv[2], wv[3], sB, vb);
#pragma unroll
        for (int f = 0; f < 4; ++f) mma_f16(o[f], va[f], va[f + 4], vb[f], vb[f + 4], pb0, pb1);
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
    for (int c2 = fail_chunk; c2 < min(n_chunks, fail_chunk + kNS); ++c2) (void)mbar_wait(&bar[c2 % kNS], (c2 / kNS) & 1);
  }

  // ── merge: per query tig, reduce l over the 8 row lanes, then the warps ──
  l_part += __shfl_xor_sync(0xffffffffu, l_part, 4);
  l_part += __shfl_xor_sync(0xffffffffu, l_part, 8);
  l_part += __shfl_xor_sync(0xffffffffu, l_part, 16);
  float* so = reinterpret_cast<float*>(smem);  // reuses the staging area once every warp is past it
  __syncthreads();
  if (gid == 0 && q_ok) {
    sm_m[warp][tig] = m_run;
    sm_l[warp][tig] = l_part;
  }
  if (q_ok) {
    float* dst = so + (warp * 4 + tig) * D;
#pragma unroll
    for (int f = 0; f < KS; ++f) {
      const int c_lo = D == 128 ? 16 * gid + f : 8 * gid + f;
      const int c_hi = D == 128 ? 16 * gid + 8 + f : 8 * gid + f + 4;
      dst[c_lo] = o[f][0] + o[f][1];
      dst[c_hi] = o[f][2] + o[f][3];
    }
  }
  __syncthreads();
  const int64_t prt = static_cast<int64_t>(bh) * a.n_splits + split;
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
        O += so[(w * 4 + i) * D + cidx] * f;
      }
    }
    a.po[(prt * QN + i) * D + cidx] = O;
    if (cidx == 0) {
      a.pm[prt * QN + i] = M;
      a.pl[prt * QN + i] = L;
    }
  }
}

}  // namespace narrow

size_t narrow_smem_bytes(const carekv_config_t& c, bool kslot) {
  const int G = c.head_dim / c.group_size;
  return static_cast<size_t>(narrow::geo(c.head_dim, G, c.k_slots_per_page, kslot).total);
}

template <int QN, int D>
cudaError_t launch_decode_narrow(DecodeArgs& a, cudaStream_t st, int n_bh) {
  const int smem = static_cast<int>(narrow_smem_bytes(a.cfg, a.kw != nullptr));
  static int attr_bytes = 0;  // per process; the attribute is per function, not per device
  if (smem > attr_bytes) {
    cudaError_t e = cudaFuncSetAttribute(narrow::decode_narrow<QN, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         smem);
    if (e != cudaSuccess) return e;
    attr_bytes = smem;
  }
  dim3 grid(n_bh, a.n_splits);
  narrow::decode_narrow<QN, D><<<grid, narrow::kWarps * 32, smem, st>>>(a);
  return cudaGetLastError();
}

#define CK_INST(QN, D) template cudaError_t launch_decode_narrow<QN, D>(DecodeArgs&, cudaStream_t, int);
CK_INST(1, 64) CK_INST(2, 64) CK_INST(4, 64)
CK_INST(1, 128) CK_INST(2, 128) CK_INST(4, 128)
#undef CK_INST

}  // namespace carekv
