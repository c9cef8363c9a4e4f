// Narrow-group split-K decode pass over packed INT3 / INT4 pages (kernel K3n,
// sm_100a): kv heads whose query group has at most 4 heads (MHA, GQA-2,
// GQA-4).
//
// Contract: like the wide pass in decode_fast.cu, every CTA streams a range
// of pages of one (sequence, kv head) and writes the logits S of every token
// and one (m, l, O) split partial.  In addition, when live combined_kvscore
// scoring is on (attention.py:167-184), it writes w = q . R_K for every
// stored K residual slot, query and token (R_K = code * slot scale over the
// slot's 32-channel group), so the router never re-reads slot payloads.
// S and w are written in the pair order of tok_pos() (decode_args.h): the
// lane that owns tokens t and t+8 stores them side by side.
//
// Orientation: tokens and channels sit on the M side of the MMAs and the
// queries on N, as 8 columns = fp16 hi and lo halves of up to 4 queries:
//     S^T [16 tok x 8]  = K_hat [16 tok x D] . Q^T [D x 8]
//     O^T [D x 8]      += V_hat^T [D x 16 tok] . P^T [16 tok x 8]
//     w^T [16 tok x 8]  = R_K [16 tok x 32] . Q_g^T [32 x 8]
// A page costs D/16 MMAs per side, each thread keeps D/4 fp32 accumulators,
// and the hi + lo split keeps ~22 significant bits of q and p, so S and O
// match an fp32 evaluation to accumulation-order rounding.  The two pages of
// a stage share one online-softmax update.
//
// Per warp: an NS-stage ring of bulk copies (cp.async.bulk + mbarrier,
// bounded waits) stages CP contiguous pages at a time: packed K and V rows,
// their int8 scale codes and the pages' K slot payloads.  Per-page metadata
// (valid rows, fp16 masters, slot groups and scales) is read 32 pages at a
// time into shared memory.  Dequantization is exact: 3-bit fields are moved
// to a mantissa bit 0..7 of an fp16 half (PRMT / SHF / LOP3), the offset
// removed with HSUB2 and the scale applied with HMUL2, i.e. fp16(code *
// scale) rounded once, as the reference dequantizes; scale codes become
// fp16(int8 * master) the same way.
#include <type_traits>
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
__host__ __device__ inline Geo geo(int D, int G, int SK, bool kslot, int bits) {
  Geo g;
  g.R = D * bits / 8;
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

// 2^x with the SFU approximation (results below 2^-126 flush to zero).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }

// 24-bit packed word at byte offset o of a staged row (bits 24..31 garbage).
__device__ __forceinline__ uint32_t word24_at(const uint8_t* row, int o) {
  const uint32_t* p = reinterpret_cast<const uint32_t*>(row + (o & ~3));
  return prmt(p[0], p[1], 0x3210 + 0x1111 * (o & 3));
}

// Magic keys of the field positions used below (DecodeArgs::dq_keys), held
// in registers: a key is both the XOR operand of the LOP3 (whose immediate
// slot holds the mask) and the subtrahend of the HSUB2.
struct Keys {
  uint32_t k0, k3, k6, n0, n4, p10, p43, p76, p22, p11, p44, p77, p55;
};
// exact half2 (code_lo, code_hi) * sig2 of two 3-bit fields at mantissa bit S
template <int S>
__device__ __forceinline__ uint32_t i3p(uint32_t t, uint32_t key, uint32_t sig2) {
  uint32_t x;  // (t & mask) ^ key in one LOP3
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(x) : "r"(t), "n"(i3_mask2(S, S)), "r"(key));
  return h2mul(h2sub(x, key), sig2);
}

// exact half2 (code_lo, code_hi) * sig2 of a 3-bit field at mantissa bit SL
// of the low half and one at bit SH of the high half
template <int SL, int SH>
__device__ __forceinline__ uint32_t i3q(uint32_t t, uint32_t key, uint32_t sig2) {
  uint32_t x;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(x) : "r"(t), "n"(i3_mask2(SL, SH)), "r"(key));
  return h2mul(h2sub(x, key), sig2);
}

// A thread's 32 INT3 channels of a K row (96 bits in x0..x2, channel i at
// bit 3i) -> 16 half2 operands, channel pairs kPairs[j], from seven 32-bit
// windows of the row: a window starting at bit b = 2 (mod 3) holds three
// fields at bits 1, 4, 7 of its low half and three at bits 0, 3, 6 of its
// high half, so one LOP3 per pair picks both fields without further shifts.
//   window  start bit  pairs (low channel, high channel)
//   x0 << 1     -1     (0,5) (1,6) (2,7)
//   x1:x0 >> 8   8     (3,8) (4,9)
//   x1:x0 >> 29 29     (10,15) (11,16) (12,17)
//   x2:x1 >> 6  38     (13,18) (14,19)
//   x2:x1 >> 27 59     (20,25) (21,26) (22,27)
//   x2 >> 4     68     (23,28) (24,29)
//   (x2 >> 24) * (1 + 2^13): channel 30 at bit 2, channel 31 at bit 18
__device__ constexpr int kPairs[16][2] = {{0, 5},   {1, 6},   {2, 7},   {3, 8},   {4, 9},   {10, 15},
                                          {11, 16}, {12, 17}, {13, 18}, {14, 19}, {20, 25}, {21, 26},
                                          {22, 27}, {23, 28}, {24, 29}, {30, 31}};
__device__ __forceinline__ void k_row32(uint32_t x0, uint32_t x1, uint32_t x2, uint32_t sig2, const Keys& K,
                                        uint32_t (&o)[16]) {
  const uint32_t w1 = x0 << 1, w2 = __funnelshift_r(x0, x1, 8), w3 = __funnelshift_r(x0, x1, 29);
  const uint32_t w4 = __funnelshift_r(x1, x2, 6), w5 = __funnelshift_r(x1, x2, 27), w6 = x2 >> 4;
  const uint32_t w7 = (x2 >> 24) * 8193u;
  o[0] = i3q<1, 0>(w1, K.p10, sig2);
  o[1] = i3q<4, 3>(w1, K.p43, sig2);
  o[2] = i3q<7, 6>(w1, K.p76, sig2);
  o[3] = i3q<1, 0>(w2, K.p10, sig2);
  o[4] = i3q<4, 3>(w2, K.p43, sig2);
  o[5] = i3q<1, 0>(w3, K.p10, sig2);
  o[6] = i3q<4, 3>(w3, K.p43, sig2);
  o[7] = i3q<7, 6>(w3, K.p76, sig2);
  o[8] = i3q<1, 0>(w4, K.p10, sig2);
  o[9] = i3q<4, 3>(w4, K.p43, sig2);
  o[10] = i3q<1, 0>(w5, K.p10, sig2);
  o[11] = i3q<4, 3>(w5, K.p43, sig2);
  o[12] = i3q<7, 6>(w5, K.p76, sig2);
  o[13] = i3q<1, 0>(w6, K.p10, sig2);
  o[14] = i3q<4, 3>(w6, K.p43, sig2);
  o[15] = i3q<2, 2>(w7, K.p22, sig2);
}

// One packed K word (codes f0..f7, 3 bits each) -> half2 operands
// (f0,f3) (f1,f4) (f2,f5) (f6,f7), every field at mantissa bit 0, 3 or 6.
__device__ __forceinline__ void k_quads(uint32_t W, uint32_t sig2, const Keys& K, uint32_t (&o)[4]) {
  const uint32_t t1 = prmt(W, W >> 9, 0x5410);         // W[0:16] | W[9:25]
  const uint32_t t2 = prmt(W >> 12, W >> 15, 0x5410);  // W[12:28] | W[15:31]
  o[0] = i3p<0>(t1, K.k0, sig2);
  o[1] = i3p<3>(t1, K.k3, sig2);
  o[2] = i3p<6>(t1, K.k6, sig2);
  o[3] = i3p<6>(t2, K.k6, sig2);
}
// The same packed word of two rows a (low halves) and b (high halves), one
// PRMT per register: f0..f2 in r[0] at bits 0, 3, 6; f3..f5 in r[1] at
// bits 1, 4, 7; f6, f7 in r[2] at bits 2, 5.
struct VSrc {
  uint32_t r[3];
};
__device__ __forceinline__ VSrc v_src(uint32_t Wa, uint32_t Wb) {
  VSrc v;
  v.r[0] = prmt(Wa, Wb, 0x5410);
  v.r[1] = prmt(Wa, Wb, 0x6521);
  v.r[2] = prmt(Wa, Wb, 0x7632);
  return v;
}
template <int F>
__device__ __forceinline__ uint32_t v_field(const VSrc& v, const Keys& K, uint32_t sig2) {
  // r[0]: f0..f2 at bits 0, 3, 6; r[1]: f3..f5 at 1, 4, 7; r[2]: f6, f7 at 2, 5
  constexpr int S = F < 3 ? 3 * F : (F < 6 ? 3 * (F - 3) + 1 : 3 * (F - 6) + 2);
  const uint32_t key = S == 0 ? K.k0 : S == 3 ? K.k3 : S == 6 ? K.k6 : S == 1 ? K.p11 : S == 4 ? K.p44 : S == 7 ? K.p77
                     : S == 2 ? K.p22 : K.p55;
  return i3p<S>(v.r[F < 3 ? 0 : (F < 6 ? 1 : 2)], key, sig2);
}

// 4-bit residual word (nibbles n0..n7) -> exact half2 codes (n0,n4) (n1,n5)
// (n2,n6) (n3,n7): nibble at mantissa bit 0 or 4, offset removed by HSUB2.
__device__ __forceinline__ void nib_quads(uint32_t u, const Keys& K, uint32_t (&o)[4]) {
  const uint32_t v = u >> 8;
  o[0] = h2sub((u & 0x000F000Fu) ^ K.n0, K.n0);
  o[1] = h2sub((u & 0x00F000F0u) ^ K.n4, K.n4);
  o[2] = h2sub((v & 0x000F000Fu) ^ K.n0, K.n0);
  o[3] = h2sub((v & 0x00F000F0u) ^ K.n4, K.n4);
}

// exact half2 (code_lo, code_hi) * sig2 of two 4-bit fields at mantissa bit S (0 or 4)
template <int S>
__device__ __forceinline__ uint32_t i4p(uint32_t t, uint32_t key, uint32_t sig2) {
  uint32_t x;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(x) : "r"(t), "n"((15u << S) | (15u << (16 + S))), "r"(key));
  return h2mul(h2sub(x, key), sig2);
}
// One packed INT4 K word (nibbles n0..n7, even channel low) -> half2 operands
// (n0,n4) (n1,n5) (n2,n6) (n3,n7).
__device__ __forceinline__ void k_quads4(uint32_t u, uint32_t sig2, const Keys& K, uint32_t (&o)[4]) {
  const uint32_t v = u >> 8;
  o[0] = i4p<0>(u, K.n0, sig2);
  o[1] = i4p<4>(u, K.n4, sig2);
  o[2] = i4p<0>(v, K.n0, sig2);
  o[3] = i4p<4>(v, K.n4, sig2);
}
// The same INT4 word of rows a (low halves) and b (high halves): byte k of
// both rows in r[k], its nibbles (channels 2k, 2k+1) at bits 0 and 4.
struct VSrc4 {
  uint32_t r[4];
};
__device__ __forceinline__ VSrc4 v_src4(uint32_t Wa, uint32_t Wb) {
  VSrc4 v;
  v.r[0] = prmt(Wa, Wb, 0x4400);
  v.r[1] = prmt(Wa, Wb, 0x5511);
  v.r[2] = prmt(Wa, Wb, 0x6622);
  v.r[3] = prmt(Wa, Wb, 0x7733);
  return v;
}
template <int F>
__device__ __forceinline__ uint32_t v_field4(const VSrc4& v, const Keys& K, uint32_t sig2) {
  return i4p<4 * (F & 1)>(v.r[F >> 1], (F & 1) ? K.n4 : K.n0, sig2);
}

// GC, SKC: scale groups per row and K slots per page fixed at compile time
// (every stage offset then folds into the instructions), or 0 = read from
// the configuration.
// KSLOT: q . R_K of the stored K slots is written (a.kw != nullptr; the
// stage then also holds the pages' slot payloads).
template <int QN, int D, int BITS, int GC, int SKC, bool KSLOT>
__global__ void __launch_bounds__(kWarps * 32, 4) decode_narrow(DecodeArgs a) {
  static_assert(BITS == 3 || BITS == 4, "narrow pass: INT3 or INT4 rows");
  constexpr int R = D * BITS / 8;
  constexpr int KS = D / 16;   // k-steps of Q.K^T = m-tiles of O^T
  constexpr int KW = D / 32;   // packed K words per thread and row
  constexpr int G4 = D / 32;   // 32-channel groups (K residual slots)
  static_assert(QN >= 1 && QN <= 4, "narrow pass: at most 4 queries per kv head");
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bars[kWarps][kNS];
  __shared__ float sm_m[kWarps][4], sm_l[kWarps][4];
  __shared__ __align__(16) float q_sm[QN][D];
  __shared__ uint2 qbs[KS][32];   // Q^T operands per k-step and lane

  const Dims d = make_dims(a.cfg);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  // consecutive CTAs share a (sequence, kv head): bh-major, split-minor
  const int bh = blockIdx.x / a.n_splits, split = blockIdx.x % a.n_splits;
  const int s = bh / d.H, h = bh % d.H, b = a.seq_begin + s;
  const int64_t lhp = d.lhp(b, a.layer, h);
  const int np = min(a.cache.num_pages[lhp], a.p_used);
  const int ca = split * a.pps, cb = min(np, ca + a.pps);
  const int n_cta = max(0, cb - ca);
  const int qv = n_cta / kWarps, rv = n_cta % kWarps;
  const int pa = ca + warp * qv + min(warp, rv);
  const int pb = pa + qv + (warp < rv ? 1 : 0);
  const int Hq = a.act_heads;   // query heads per activation row
  const int G = GC > 0 ? GC : d.G, SK = SKC > 0 ? SKC : d.SK;
  constexpr bool kslot = KSLOT;
  const Geo g = geo(D, G, SK, kslot, BITS);
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

  // bulk copies of chunk c (pages pa + 2c, pa + 2c + 1); sources are
  // recomputed from the arguments on every issue (one lane, once per chunk)
  const int n_chunks = (pb - pa + kCP - 1) / kCP;
  // the packed pages are read once (evict first); S and q . R_K are read
  // back by the router right after this pass (evict last)
  const uint64_t pol_stream = l2_evict_first(), pol_keep = l2_evict_last();
  auto issue = [&](int c) {
    const int p = pa + c * kCP;
    const int n = min(kCP, pb - p);
    const int slot = c % kNS;
    uint8_t* st = wsm + slot * g.stage;
    uint64_t* br = &bar[slot];
    const int64_t pg = page0 + p;
    const uint32_t cbytes = n * kPage * R, sbytes = n * kPage * G;
    const uint32_t slbytes = kslot ? n * SK * 256 : 0;
    mbar_expect_tx(br, 2 * cbytes + 2 * sbytes + slbytes);
    bulk_g2s_pol(st, a.cache.k_codes + pg * (kPage * R), cbytes, br, pol_stream);
    bulk_g2s_pol(st + g.vOff, a.cache.v_codes + pg * (kPage * R), cbytes, br, pol_stream);
    bulk_g2s_pol(st + g.ksOff, reinterpret_cast<const int8_t*>(a.cache.k_scale) + pg * kPage * G, sbytes, br, pol_stream);
    bulk_g2s_pol(st + g.vsOff, reinterpret_cast<const int8_t*>(a.cache.v_scale) + pg * kPage * G, sbytes, br, pol_stream);
    if (slbytes) bulk_g2s_pol(st + g.slOff, a.cache.k_slot_data + pg * SK * 256, slbytes, br, pol_stream);
  };
  if (lane == 0)
    for (int c = 0; c < min(kNS, n_chunks); ++c) issue(c);

  // ── queries (fp32) in shared memory, then the Q^T operands ──
  for (int x = threadIdx.x; x < QN * D; x += blockDim.x)
    q_sm[x / D][x % D] = load_act(a.q, (static_cast<int64_t>(s) * Hq + h * QN) * D + x, a.dt);
  __syncthreads();
  // column n = query n/2, half n%2 (0 = hi, 1 = lo)
  const int qi = gid >> 1, part = gid & 1;
  auto qp = [&](int c) -> float {
    if (qi >= QN) return 0.f;
    const float x = q_sm[qi][c];
    const float hi = __half2float(__float2half_rn(x));
    return part ? x - hi : hi;
  };
  // K side: thread tig owns channels tig*D/4 .. +D/4 (KW packed words); word
  // i feeds k-steps 2i and 2i+1 (channel pairs as the k_quads / k_quads4
  // operands pair them).  Built once per CTA: warp w fills the k-steps of the
  // words i with i % kWarps == w; every warp then loads all of them.
  constexpr bool kRow32 = BITS == 3 && D == 128;   // k_row32 operand order
  if constexpr (kRow32) {        // k-step ks takes channel pairs 2ks, 2ks+1 of kPairs
    for (int ks = warp; ks < KS; ks += kWarps) {
      const int c = tig * 32;
      qbs[ks][lane] = make_uint2(pack_h2(qp(c + kPairs[2 * ks][0]), qp(c + kPairs[2 * ks][1])),
                                 pack_h2(qp(c + kPairs[2 * ks + 1][0]), qp(c + kPairs[2 * ks + 1][1])));
    }
  }
  for (int i = warp; i < (kRow32 ? 0 : KW); i += kWarps) {
    const int c = tig * (D / 4) + 8 * i;
    if constexpr (BITS == 3) {   // k_quads: (f0,f3) (f1,f4) | (f2,f5) (f6,f7)
      qbs[2 * i][lane] = make_uint2(pack_h2(qp(c + 0), qp(c + 3)), pack_h2(qp(c + 1), qp(c + 4)));
      qbs[2 * i + 1][lane] = make_uint2(pack_h2(qp(c + 2), qp(c + 5)), pack_h2(qp(c + 6), qp(c + 7)));
    } else {                     // k_quads4: (n0,n4) (n1,n5) | (n2,n6) (n3,n7)
      qbs[2 * i][lane] = make_uint2(pack_h2(qp(c + 0), qp(c + 4)), pack_h2(qp(c + 1), qp(c + 5)));
      qbs[2 * i + 1][lane] = make_uint2(pack_h2(qp(c + 2), qp(c + 6)), pack_h2(qp(c + 3), qp(c + 7)));
    }
  }
  // slot operands per 32-channel group: thread tig owns the group's channels
  // 8*tig .. +8 (one nibble word per token); k-step 0 takes (n0,n4) (n1,n5),
  // k-step 1 (n2,n6) (n3,n7)
  if (kslot) {
    for (int x = threadIdx.x; x < G4 * 2 * 32; x += blockDim.x) {
      const int grp = x / 64, ks = (x / 32) % 2, ln = x % 32;
      const int lq = (ln >> 2) >> 1, lp = (ln >> 2) & 1, c0 = grp * 32 + 8 * (ln & 3) + 2 * ks;
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      if (lq < QN) {
        const int cs[4] = {c0, c0 + 4, c0 + 1, c0 + 5};
        for (int e = 0; e < 4; ++e) {
          const float xq = q_sm[lq][cs[e]];
          const float hi = __half2float(__float2half_rn(xq));
          v[e] = lp ? xq - hi : hi;
        }
      }
      qs[x] = make_uint2(pack_h2(v[0], v[1]), pack_h2(v[2], v[3]));
    }
  }
  __syncthreads();
  uint32_t qb[KS][2];
#pragma unroll
  for (int kb = 0; kb < KS; ++kb) {
    const uint2 v = qbs[kb][lane];
    qb[kb][0] = v.x;
    qb[kb][1] = v.y;
  }

  const Keys KY = {a.dq_keys[0], a.dq_keys[1],  a.dq_keys[2],  a.dq_keys[3],  a.dq_keys[4],
                   a.dq_keys[5], a.dq_keys[6],  a.dq_keys[7],  a.dq_keys[8],  a.dq_keys[9],
                   a.dq_keys[10], a.dq_keys[11], a.dq_keys[12]};
  float o[KS][4];
#pragma unroll
  for (int j = 0; j < KS; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_run = -INFINITY, l_part = 0.f;
  const bool q_ok = tig < QN;
  float* Srow = a.S + (static_cast<int64_t>(bh) * QN + tig) * a.p_used * kPage + 2 * gid;
  float* Wrow = kslot ? a.kw + (static_cast<int64_t>(bh) * QN + tig) * KG * kPage + 2 * gid : nullptr;

  // V side: thread gid owns packed words (D=128) 2gid, 2gid+1 / (D=64) gid
  constexpr int VB = (D == 128 ? 2 : 1) * BITS;   // bytes of the thread's V words: one 8-channel word = BITS bytes
  const int vo = VB * gid;
  const int vbase = vo & ~3, voff = vo & 3;
  const uint32_t vsel_l = 0x3210 + 0x1111 * voff;
  const uint32_t vsel_h = (0x3210 + 0x1111 * (voff + 3)) & 0x7777;
  const int gsz = GC > 0 ? D / GC : d.gsize;
  const int gk = (tig * (D / 4)) / gsz;                  // K scale group of the thread's channels
  const int gv = ((D == 128 ? 16 : 8) * gid) / gsz;      // V scale group
  const int ra = 2 * tig;                                 // V rows ra, ra+1, ra+8, ra+9
  const int src_a = 8 * tig + qi, src_b = src_a + 4;
  const int ko0 = gid * R + (D / 4) * BITS / 8 * tig, ko8 = ko0 + 8 * R;   // thread's K channel block
  const int kso0 = gid * G + gk, kso8 = (gid + 8) * G + gk;
  const int vso0 = ra * G + gv, vso1 = (ra + 1) * G + gv, vso2 = (ra + 8) * G + gv, vso3 = (ra + 9) * G + gv;

  // logits of one staged page for rows gid, gid+8
  auto k_side = [&](const uint8_t* st, int pp, uint32_t km2, float& s0, float& s1) {
    const uint8_t* kc = st + pp * kPage * R;
    const uint8_t* ks = st + g.ksOff + pp * kPage * G;
    const uint32_t sig = i8_scale_pair(static_cast<uint32_t>(ks[kso0]) | (static_cast<uint32_t>(ks[kso8]) << 16), km2);
    const uint32_t sig0 = prmt(sig, sig, 0x1010), sig8 = prmt(sig, sig, 0x3232);
    if constexpr (kRow32) {
      uint32_t p0[16], p8[16];
      k_row32(lds32(kc + ko0), lds32(kc + ko0 + 4), lds32(kc + ko0 + 8), sig0, KY, p0);
      k_row32(lds32(kc + ko8), lds32(kc + ko8 + 4), lds32(kc + ko8 + 8), sig8, KY, p8);
      float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int ks = 0; ks < KS; ++ks)
        mma_f16(acc[ks & 1], p0[2 * ks], p8[2 * ks], p0[2 * ks + 1], p8[2 * ks + 1], qb[ks][0], qb[ks][1]);
      s0 = __fmul_rn((acc[0][0] + acc[1][0]) + (acc[0][1] + acc[1][1]), a.sf);
      s1 = __fmul_rn((acc[0][2] + acc[1][2]) + (acc[0][3] + acc[1][3]), a.sf);
      return;
    }
    uint32_t w0[KW], w8[KW];
    if constexpr (BITS == 4) {
#pragma unroll
      for (int i = 0; i < KW; ++i) {
        w0[i] = lds32(kc + ko0 + 4 * i);
        w8[i] = lds32(kc + ko8 + 4 * i);
      }
    } else if constexpr (D == 128) {
      const uint32_t x0 = lds32(kc + ko0), x1 = lds32(kc + ko0 + 4), x2 = lds32(kc + ko0 + 8);
      const uint32_t y0 = lds32(kc + ko8), y1 = lds32(kc + ko8 + 4), y2 = lds32(kc + ko8 + 8);
      w0[0] = x0; w0[1] = prmt(x0, x1, 0x6543); w0[2] = prmt(x1, x2, 0x5432); w0[3] = x2 >> 8;
      w8[0] = y0; w8[1] = prmt(y0, y1, 0x6543); w8[2] = prmt(y1, y2, 0x5432); w8[3] = y2 >> 8;
    } else {
#pragma unroll
      for (int i = 0; i < KW; ++i) {
        w0[i] = word24_at(kc + gid * R, 6 * tig + 3 * i);
        w8[i] = word24_at(kc + (gid + 8) * R, 6 * tig + 3 * i);
      }
    }
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int i = 0; i < KW; ++i) {
      uint32_t p0[4], p8[4];
      if constexpr (BITS == 4) {
        k_quads4(w0[i], sig0, KY, p0);
        k_quads4(w8[i], sig8, KY, p8);
      } else {
        k_quads(w0[i], sig0, KY, p0);
        k_quads(w8[i], sig8, KY, p8);
      }
      mma_f16(acc[i & 1], p0[0], p8[0], p0[1], p8[1], qb[2 * i][0], qb[2 * i][1]);
      mma_f16(acc[i & 1], p0[2], p8[2], p0[3], p8[3], qb[2 * i + 1][0], qb[2 * i + 1][1]);
    }
    s0 = __fmul_rn((acc[0][0] + acc[1][0]) + (acc[0][1] + acc[1][1]), a.sf);
    s1 = __fmul_rn((acc[0][2] + acc[1][2]) + (acc[0][3] + acc[1][3]), a.sf);
  };

  // w = q . R_K of the page's stored K slots
  auto slot_side = [&](const uint8_t* st, int pp, int p, int mi, int nv) {
    if (nv == 0) return;
    for (int j = 0; j < SK; ++j) {
      const int grp = m_grp[mi * SK + j];
      if (grp < 0 || grp >= G4) continue;
      const uint8_t* sl = st + g.slOff + (pp * SK + j) * 256 + 4 * tig;
      uint32_t n0[4], n8[4];
      nib_quads(lds32(sl + gid * 16), KY, n0);
      nib_quads(lds32(sl + (gid + 8) * 16), KY, n8);
      const uint2 b0 = qs[(grp * 2 + 0) * 32 + lane];
      const uint2 b1 = qs[(grp * 2 + 1) * 32 + lane];
      float cw[4] = {0.f, 0.f, 0.f, 0.f};
      mma_f16(cw, n0[0], n8[0], n0[1], n8[1], b0.x, b0.y);
      mma_f16(cw, n0[2], n8[2], n0[3], n8[3], b1.x, b1.y);
      const float rs = m_rs[mi * SK + j];
      if (q_ok)
        st_f2_pol(Wrow + (static_cast<int64_t>(p) * SK + j) * kPage, __fmul_rn(cw[0] + cw[1], rs),
                  __fmul_rn(cw[2] + cw[3], rs), pol_keep);
    }
  };

  // O^T += V_hat^T . P^T for one staged page
  auto v_side = [&](const uint8_t* st, int pp, uint32_t vm2, uint32_t pb0, uint32_t pb1) {
    const uint8_t* vc = st + g.vOff + pp * kPage * R;
    const uint8_t* vs = st + g.vsOff + pp * kPage * G;
    const uint32_t sA = i8_scale_pair(static_cast<uint32_t>(vs[vso0]) | (static_cast<uint32_t>(vs[vso1]) << 16), vm2);
    const uint32_t sB = i8_scale_pair(static_cast<uint32_t>(vs[vso2]) | (static_cast<uint32_t>(vs[vso3]) << 16), vm2);
    if constexpr (BITS == 4) {
      if constexpr (D == 128) {
        uint32_t wl[4], wh[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const uint2 w2 = *reinterpret_cast<const uint2*>(vc + (ra + (r & 1) + 8 * (r >> 1)) * R + vo);
          wl[r] = w2.x;
          wh[r] = w2.y;
        }
        const VSrc4 x0 = v_src4(wl[0], wl[1]), x1 = v_src4(wh[0], wh[1]);
        const VSrc4 x2 = v_src4(wl[2], wl[3]), x3 = v_src4(wh[2], wh[3]);
#define CK_VF(F) \
  mma_f16(o[F], v_field4<F>(x0, KY, sA), v_field4<F>(x1, KY, sA), v_field4<F>(x2, KY, sB), v_field4<F>(x3, KY, sB), pb0, pb1);
        CK_VF(0) CK_VF(1) CK_VF(2) CK_VF(3) CK_VF(4) CK_VF(5) CK_VF(6) CK_VF(7)
#undef CK_VF
      } else {
        uint32_t wv[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) wv[r] = lds32(vc + (ra + (r & 1) + 8 * (r >> 1)) * R + vo);
        const VSrc4 x0 = v_src4(wv[0], wv[1]), x1 = v_src4(wv[2], wv[3]);
#define CK_VF(F)                                                                                                   \
  mma_f16(o[F], v_field4<F>(x0, KY, sA), v_field4<F + 4>(x0, KY, sA), v_field4<F>(x1, KY, sB), v_field4<F + 4>(x1, KY, sB), \
          pb0, pb1);
        CK_VF(0) CK_VF(1) CK_VF(2) CK_VF(3)
#undef CK_VF
      }
    } else if constexpr (D == 128) {
      uint32_t wl[4], wh[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const uint8_t* rp = vc + (ra + (r & 1) + 8 * (r >> 1)) * R + vbase;
        const uint32_t lo = lds32(rp), hi = lds32(rp + 4);
        wl[r] = prmt(lo, hi, vsel_l);
        wh[r] = prmt(lo, hi, vsel_h);
      }
      const VSrc x0 = v_src(wl[0], wl[1]), x1 = v_src(wh[0], wh[1]);
      const VSrc x2 = v_src(wl[2], wl[3]), x3 = v_src(wh[2], wh[3]);
#define CK_VF(F) \
  mma_f16(o[F], v_field<F>(x0, KY, sA), v_field<F>(x1, KY, sA), v_field<F>(x2, KY, sB), v_field<F>(x3, KY, sB), pb0, pb1);
      CK_VF(0) CK_VF(1) CK_VF(2) CK_VF(3) CK_VF(4) CK_VF(5) CK_VF(6) CK_VF(7)
#undef CK_VF
    } else {
      uint32_t wv[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) wv[r] = word24_at(vc + (ra + (r & 1) + 8 * (r >> 1)) * R, vo);
      const VSrc x0 = v_src(wv[0], wv[1]), x1 = v_src(wv[2], wv[3]);
#define CK_VF(F)                                                                                           \
  mma_f16(o[F], v_field<F>(x0, KY, sA), v_field<F + 4>(x0, KY, sA), v_field<F>(x1, KY, sB), v_field<F + 4>(x1, KY, sB), \
          pb0, pb1);
      CK_VF(0) CK_VF(1) CK_VF(2) CK_VF(3)
#undef CK_VF
    }
  };

  // P^T operands of one page: tokens 2tig, 2tig+1 | 2tig+8, 2tig+9 of query
  // qi, from the (hi, lo) pairs of the lanes that computed them
  auto p_operands = [&](float pr0, float pr1, uint32_t& pb0, uint32_t& pb1) {
    const uint32_t HI = pack_h2(pr0, pr1);
    const float2 hf = __half22float2(*reinterpret_cast<const __half2*>(&HI));
    const uint32_t LO = pack_h2(pr0 - hf.x, pr1 - hf.y);
    const uint32_t T0 = prmt(HI, LO, 0x5410), T1 = prmt(HI, LO, 0x7632);  // (hi, lo) of token gid / gid+8
    const uint32_t xa = __shfl_sync(0xffffffffu, T0, src_a), xb = __shfl_sync(0xffffffffu, T0, src_b);
    const uint32_t ya = __shfl_sync(0xffffffffu, T1, src_a), yb = __shfl_sync(0xffffffffu, T1, src_b);
    const uint32_t sel = part ? 0x7632u : 0x5410u;
    pb0 = prmt(xa, xb, sel);
    pb1 = prmt(ya, yb, sel);
  };

  bool failed = false;
  int fail_chunk = n_chunks;
  int slot = 0;        // c % kNS
  uint32_t phase = 0;  // (c / kNS) & 1
  for (int c = 0; c < n_chunks; ++c) {
    const int pbase = pa + c * kCP;
    const int mi = (pbase - pa) & (kWin - 1);
    if (mi == 0) {
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
    if (!mbar_wait(&bar[slot], phase)) {
      failed = true;
      fail_chunk = c;
      if (lane == 0) atomicOr(a.cache.error_flag, 4);
      break;
    }
    const uint8_t* st = wsm + slot * g.stage;
    // a full stage (two pages) runs as one straight-line block; the odd
    // last page of a range takes the one-page form
    auto stage = [&](auto npc) {
      constexpr bool two = decltype(npc)::value == 2;
      const int nv0 = m_valid[mi], nv1 = two ? m_valid[mi + 1] : 0;

      // ── logits of both pages ──
      float s00, s01, s10 = 0.f, s11 = 0.f;
      k_side(st, 0, m_km[mi], s00, s01);
      if constexpr (two) k_side(st, 1, m_km[mi + 1], s10, s11);
      if (q_ok) {
        st_f2_pol(Srow + static_cast<int64_t>(pbase) * kPage, s00, s01, pol_keep);
        if constexpr (two) st_f2_pol(Srow + static_cast<int64_t>(pbase + 1) * kPage, s10, s11, pol_keep);
      }
      if (kslot) {
        slot_side(st, 0, pbase, mi, nv0);
        if constexpr (two) slot_side(st, 1, pbase + 1, mi + 1, nv1);
      }

      // ── online softmax for query tig over the stage's tokens ──
      const bool v00 = gid < nv0, v01 = gid + 8 < nv0, v10 = gid < nv1, v11 = gid + 8 < nv1;
      float pmax = fmaxf(fmaxf(v00 ? s00 : -INFINITY, v01 ? s01 : -INFINITY),
                         fmaxf(v10 ? s10 : -INFINITY, v11 ? s11 : -INFINITY));
      pmax = fmaxf(pmax, __shfl_xor_sync(0xffffffffu, pmax, 4));
      pmax = fmaxf(pmax, __shfl_xor_sync(0xffffffffu, pmax, 8));
      pmax = fmaxf(pmax, __shfl_xor_sync(0xffffffffu, pmax, 16));
      if (__any_sync(0xffffffffu, pmax > m_run)) {
        const float m_new = fmaxf(m_run, pmax);
        const float alpha = m_new > m_run ? (m_run == -INFINITY ? 0.f : ex2((m_run - m_new) * kLog2e)) : 1.f;
        l_part *= alpha;
#pragma unroll
        for (int j = 0; j < KS; ++j) {
          o[j][0] *= alpha; o[j][1] *= alpha; o[j][2] *= alpha; o[j][3] *= alpha;
        }
        m_run = m_new;
      }
      const float mb = m_run * kLog2e;
      const float p00 = v00 ? ex2(fmaf(s00, kLog2e, -mb)) : 0.f;
      const float p01 = v01 ? ex2(fmaf(s01, kLog2e, -mb)) : 0.f;
      const float p10 = v10 ? ex2(fmaf(s10, kLog2e, -mb)) : 0.f;
      const float p11 = v11 ? ex2(fmaf(s11, kLog2e, -mb)) : 0.f;
      l_part += (p00 + p01) + (p10 + p11);

      // ── values ──
      uint32_t pb0, pb1;
      p_operands(p00, p01, pb0, pb1);
      v_side(st, 0, m_vm[mi], pb0, pb1);
      if constexpr (two) {
        p_operands(p10, p11, pb0, pb1);
        v_side(st, 1, m_vm[mi + 1], pb0, pb1);
      }
    };
    if (pbase + 1 < pb)
      stage(std::integral_constant<int, 2>{});
    else
      stage(std::integral_constant<int, 1>{});
    __syncwarp();
    if (lane == 0 && c + kNS < n_chunks) {
      fence_proxy_async();
      issue(c + kNS);
    }
    if (++slot == kNS) {
      slot = 0;
      phase ^= 1u;
    }
  }
  if (failed && lane == 0) {
    // let the copies already issued land (bounded) before the staging area
    // is reused or the CTA exits
    for (int c2 = fail_chunk; c2 < min(n_chunks, fail_chunk + kNS); ++c2)
      (void)mbar_wait(&bar[c2 % kNS], (c2 / kNS) & 1);
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
  return static_cast<size_t>(narrow::geo(c.head_dim, G, c.k_slots_per_page, kslot, c.base_bits).total);
}

template <int QN, int D, int BITS, int GC, int SKC, bool KSLOT>
static cudaError_t launch_narrow_ks(DecodeArgs& a, cudaStream_t st, int n_bh) {
  const int smem = static_cast<int>(narrow_smem_bytes(a.cfg, KSLOT));
  static int attr_bytes = 0;  // per process; the attribute is per function, not per device
  if (smem > attr_bytes) {
    cudaError_t e = cudaFuncSetAttribute(narrow::decode_narrow<QN, D, BITS, GC, SKC, KSLOT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr_bytes = smem;
  }
  narrow::decode_narrow<QN, D, BITS, GC, SKC, KSLOT><<<n_bh * a.n_splits, narrow::kWarps * 32, smem, st>>>(a);
  return cudaGetLastError();
}

template <int QN, int D, int BITS, int GC, int SKC>
static cudaError_t launch_narrow_kernel(DecodeArgs& a, cudaStream_t st, int n_bh) {
  return a.kw != nullptr ? launch_narrow_ks<QN, D, BITS, GC, SKC, true>(a, st, n_bh)
                         : launch_narrow_ks<QN, D, BITS, GC, SKC, false>(a, st, n_bh);
}

// 32-channel scale groups with one or two K slots per page (store budgets
// up to ~6 % at D = 128) take the compile-time layout; other layouts read G
// and SK from the configuration.
template <int QN, int D, int BITS>
static cudaError_t launch_narrow_bits(DecodeArgs& a, cudaStream_t st, int n_bh) {
  a.s_perm = 1;
  if (a.cfg.group_size == 32 && a.cfg.k_slots_per_page == 1)
    return launch_narrow_kernel<QN, D, BITS, D / 32, 1>(a, st, n_bh);
  if (a.cfg.group_size == 32 && a.cfg.k_slots_per_page == 2)
    return launch_narrow_kernel<QN, D, BITS, D / 32, 2>(a, st, n_bh);
  return launch_narrow_kernel<QN, D, BITS, 0, 0>(a, st, n_bh);
}

template <int QN, int D>
cudaError_t launch_decode_narrow(DecodeArgs& a, cudaStream_t st, int n_bh) {
  return a.cfg.base_bits == 4 ? launch_narrow_bits<QN, D, 4>(a, st, n_bh) : launch_narrow_bits<QN, D, 3>(a, st, n_bh);
}

#define CK_INST(QN, D) template cudaError_t launch_decode_narrow<QN, D>(DecodeArgs&, cudaStream_t, int);
CK_INST(1, 64) CK_INST(2, 64) CK_INST(4, 64)
CK_INST(1, 128) CK_INST(2, 128) CK_INST(4, 128)
#undef CK_INST

}  // namespace carekv
