// Route + correct (kernels K4 + K2) for QN query heads of one (sequence,
// kv head), as a device function of NW warps; route_kernel2 (route.cu) runs
// it with one CTA per (sequence, kv head, query head) after every split-K
// pass, and with one CTA per (position, kv head) for the prefill correction.
//
//  1. merge the split-K partials into O_base, M and L;
//  2. score every stored residual slot: K slots with combined_kvscore
//     (attention.py:167-184) -- from the q . R_K the narrow pass wrote, or on
//     the tensor cores here, one warp per slot -- or the sketch proxy
//     (attention.py:718-725); V slots with block attention mass x error
//     norm (attention.py:787-790), one thread per slot;
//  3. normalise per query (attention.py:830-844) and select the joint or
//     separate top-k (attention.py:856-875): a threshold from every warp's
//     r-th best lane maximum leaves a few dozen candidates that one warp sorts
//     (bitonic, ties to the lower grid index); when more survive, every warp
//     keeps a running top-32 and warp 0 merges the lists;
//  4. apply the exact softmax renormalisation (attention.py:96-118, in the
//     sparse form dO = (O + sum_S A(e^ds-1)V + sum_V A e^ds R_V) /
//     (1 + sum_S A(e^ds-1)) - O) or the linear form, one selected page or slot
//     per warp, packed rows staged in shared memory and decoded a word (8
//     channels) per lane, and write O = O_base + dO.
//
// Grid index: K entries (page, slot j) at p*SK + j, then V entries at
// KG + p*SV + j; slot tables keep groups in ascending order, so the index
// order is the reference's (page, group) order with K before V.
#pragma once
#include "common.cuh"
#include "decode_args.h"
#include "ptx.cuh"

namespace carekv {

constexpr int kRSel = 32;     // selected items per apply round (a selection may hold more)
constexpr int kRStg = 12 * 1024;   // apply staging bytes per CTA
constexpr float kREps = 1e-6f;
constexpr float kIllNorm = 0.01f;   // new-normaliser bound below which the direct exact form runs
constexpr float kRL2e = 1.4426950408889634f;

// 2^x with the SFU approximation (relative error ~2^-22; results below
// 2^-126 flush to zero): attention weights A = 2^((s - M) log2 e) / L.
__device__ __forceinline__ float rex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Selection order (score descending, grid index ascending) as one unsigned
// 64-bit key: the score's bits made order-preserving in the high word (-0
// folded onto +0), the complemented index in the low word, so a larger key
// ranks first and every compare-exchange is a branch-free min / max.
__device__ __forceinline__ uint64_t rkey(float s, int i) {
  uint32_t b = __float_as_uint(__fadd_rn(s, 0.0f));
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (static_cast<uint64_t>(b) << 32) | static_cast<uint32_t>(~i);
}
__device__ __forceinline__ float rkey_score(uint64_t k) {
  uint32_t b = static_cast<uint32_t>(k >> 32);
  b = (b & 0x80000000u) ? (b & 0x7fffffffu) : ~b;
  return __uint_as_float(b);
}
__device__ __forceinline__ int rkey_index(uint64_t k) { return static_cast<int>(~static_cast<uint32_t>(k)); }
__device__ __forceinline__ uint64_t rshfl_xor(uint64_t k, int m) {
  const uint32_t lo = __shfl_xor_sync(0xffffffffu, static_cast<uint32_t>(k), m);
  const uint32_t hi = __shfl_xor_sync(0xffffffffu, static_cast<uint32_t>(k >> 32), m);
  return (static_cast<uint64_t>(hi) << 32) | lo;
}
__device__ __forceinline__ uint64_t rshfl(uint64_t k, int src) {
  const uint32_t lo = __shfl_sync(0xffffffffu, static_cast<uint32_t>(k), src);
  const uint32_t hi = __shfl_sync(0xffffffffu, static_cast<uint32_t>(k >> 32), src);
  return (static_cast<uint64_t>(hi) << 32) | lo;
}
// One compare-exchange of a bitonic network on keys held one per lane;
// pos = the key's position in the sequence.
__device__ __forceinline__ uint64_t rcx(uint64_t k, int pos, int size, int stride) {
  const uint64_t o = rshfl_xor(k, stride);
  const bool keep_max = ((pos & stride) == 0) == ((pos & size) == 0);
  return keep_max ? (o > k ? o : k) : (o < k ? o : k);
}
// Sort up to 64 keys held two per lane (positions lane and lane + 32),
// best first: bitonic network on the warp's shuffles.
__device__ __forceinline__ void rsort64(uint64_t& k0, uint64_t& k1, int lane) {
#pragma unroll
  for (int size = 2; size <= 64; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      if (stride == 32) {
        const uint64_t hi = k0 > k1 ? k0 : k1, lo = k0 > k1 ? k1 : k0;
        k0 = hi;
        k1 = lo;
      } else {
        k0 = rcx(k0, lane, size, stride);
        k1 = rcx(k1, lane + 32, size, stride);
      }
    }
  }
}
// Merge two descending 32-lists held one key per lane (lane 0 best): keep
// the better of run[l] and blk[31 - l] (a bitonic sequence holding the top
// 32 of both) and sort it descending.
__device__ __forceinline__ uint64_t rmerge32(uint64_t run, uint64_t blk, int lane) {
  const uint64_t o = rshfl(blk, 31 - lane);
  run = o > run ? o : run;
#pragma unroll
  for (int stride = 16; stride > 0; stride >>= 1) run = rcx(run, lane, 64, stride);
  return run;
}

// 24-bit packed word at byte offset o of a staged row (bits 24..31 garbage).
__device__ __forceinline__ uint32_t rword24(const uint8_t* row, int o) {
  const uint32_t* p = reinterpret_cast<const uint32_t*>(row + (o & ~3));
  return prmt(p[0], p[1], 0x3210 + 0x1111 * (o & 3));
}
// acc[j] += cf * fp16(code_j * sigma) for the 8 channels of packed INT3 word w
// of a row (exact fp16 dequantization: field -> mantissa, HSUB2, HMUL2)
__device__ __forceinline__ void acc_int3_word(const uint8_t* row, int w, uint32_t sig2, float cf, float (&acc)[8]) {
  const uint32_t W = rword24(row, 3 * w);
  const uint32_t t = prmt(W, W << 13, 0x7610);         // low W[0:16], high W[3:19]
  const uint32_t t2 = prmt(W >> 12, W << 1, 0x7610);   // low W[12:28], high W[15:31]
  const uint32_t h[4] = {i3_pair<0, 0>(t, sig2), i3_pair<6, 6>(t, sig2), i3_pair<0, 0>(t2, sig2),
                         i3_pair<6, 6>(t2, sig2)};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h[k]));
    acc[2 * k] = fmaf(cf, f.x, acc[2 * k]);
    acc[2 * k + 1] = fmaf(cf, f.y, acc[2 * k + 1]);
  }
}
// acc[j] += c * code_j for the 8 nibbles of a 4-bit residual word
__device__ __forceinline__ void acc_nib_word(uint32_t u, float c, float (&acc)[8]) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t hk = nib_pair(u, k);
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hk));
    acc[2 * k] = fmaf(c, f.x, acc[2 * k]);
    acc[2 * k + 1] = fmaf(c, f.y, acc[2 * k + 1]);
  }
}

// Direct exact form: o2 += A_t V_hat_t and z2 += A_t over the valid rows of
// one page for the lane's channels cb .. cb+3, the rows and scales of the
// page at `rows` / `scales` (shared or global memory, indexed as the arena
// does: row t at t*R, scale of (t, group) at t*G + group), the page's token
// weights on lanes 0..15 of At.  Lane l holds channels 4l of every row; with
// D = 64 the two half-warps take alternate rows instead (lane l: channels
// 4 (l mod 16) of the rows of parity l / 16; the caller adds the halves).
// Rows are fetched four at a time per warp.
struct DirectLane {
  int cb, b0, wsh;
  int rs, half;   // rows side by side in the warp (1 or 2), the lane's row parity
  bool cl, two;
  uint32_t cmask, csign;
};
template <int RS>
__device__ __forceinline__ void direct_rows_rs(const Dims& d, int dt, const DirectLane& dl, const uint8_t* rows,
                                               const void* scales, float vm, int nv, float At, float (&o2)[4],
                                               float& z2) {
  constexpr int NU = 4 / RS;   // rows of the lane per step of 4
#pragma unroll 1
  for (int t0 = 0; t0 < kPage; t0 += 4) {
    if (t0 >= nv) break;
    uint32_t wlo[NU], whi[NU];
    float vs[NU];
#pragma unroll
    for (int u = 0; u < NU; ++u) {
      const int t = t0 + u * RS + dl.half;
      const uint32_t* row = reinterpret_cast<const uint32_t*>(rows + t * d.R);
      wlo[u] = dl.cl ? row[dl.b0 >> 5] : 0u;
      whi[u] = dl.cl && dl.two ? row[(dl.b0 >> 5) + 1] : 0u;
      vs[u] = !dl.cl ? 0.f
                     : (d.kivi ? reinterpret_cast<const float*>(scales)[t * d.G]
                               : read_scale(scales, t * d.G + dl.cb / d.gsize, d.scale_mode, vm));
    }
#pragma unroll
    for (int u = 0; u < NU; ++u) {
      // the warp's first row of the step is valid (uniform); the lane's row
      // may lie past the page's rows
      if (t0 + u * RS >= nv) break;
      const int t = t0 + u * RS + dl.half;
      const float A = __shfl_sync(0xffffffffu, At, t);
      if (t < nv) {
        z2 += A;
        const uint32_t win = __funnelshift_r(wlo[u], whi[u], dl.wsh);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t cu = (win >> (k * d.bits)) & dl.cmask;
          const int cv = static_cast<int>(cu) - static_cast<int>((cu & dl.csign) << 1);
          const float vh = d.kivi ? f16r(kivi_hat(cv, vs[u], dt)) : f16r(__fmul_rn(static_cast<float>(cv), vs[u]));
          o2[k] = fmaf(A, vh, o2[k]);
        }
      }
    }
  }
}
__device__ __forceinline__ void direct_rows(const Dims& d, int dt, const DirectLane& dl, const uint8_t* rows,
                                            const void* scales, float vm, int nv, float At, float (&o2)[4],
                                            float& z2) {
  if (dl.rs == 2) direct_rows_rs<2>(d, dt, dl, rows, scales, vm, nv, At, o2, z2);
  else direct_rows_rs<1>(d, dt, dl, rows, scales, vm, nv, At, o2, z2);
}

// Scratch of one routing CTA: QN queries, NW warps.
template <int QN, int NW>
struct RouteSmem {
  float Q[QN][128];
  float O[QN][128];
  float M[QN], invL[QN], L[QN], mlb[QN];   // mlb = M log2(e) + log2(L)
  float red[NW][QN], red2[NW][QN];
  float nk[QN], nv[QN];
  int sel[QN][kRSel];            // the first kRSel selected entries, or the current apply round
  int nsel[QN];                  // selected entries per query (any count up to the grid size)
  int hist[256];                 // radix-select histogram (selections above kRSel)
  int rsel[4];                   // radix select: digit, remaining count; scan totals
  int scan[NW];
  // per-warp top-32 lists of the selection; the prefilter uses the first NW
  // entries for thresholds and entries 32..95 for candidates
  float gv[NW * 32 > 96 ? NW * 32 : 96];
  int gi[NW * 32 > 96 ? NW * 32 : 96];
  int gcount;
  float ds[kRSel][kPage];         // wK (unscaled q.R_K) per selected K page and token
  int kp_page[kRSel], kp_mask[kRSel], kp_nv[kRSel];
  float kp_vm[kRSel];
  int vsel[kRSel], vs_t0[kRSel], vs_t1[kRSel];
  float vs_rs[kRSel];
  int ioff[2 * kRSel], bnd[2 * kRSel + 1], nb;
  uint64_t stg_bar;
  float acc[NW][128];
  float z[NW];
  float acc2[NW][128];   // attention-weighted V of the tokens outside the selected K pages
  float z2[NW];          // and their attention mass (direct form of an ill-conditioned query)
  int ill;
  union {
    __align__(16) uint32_t qfrag[4][2][32][4];  // A fragments of q_hi / q_lo per channel group and k-step (scoring)
    __align__(16) uint8_t stg[kRStg];           // staged items (apply)
  };
  float stage_sc[NW][16 * 4];           // the page's V scales (fp16 values)
  float coef[NW][kPage];
  int cnt_k, cnt_v, ntot, any_k, nkp, nvs;
  float mshift;
  float zS;              // sum over the selected K pages' tokens of A (e^ds - 1)
  float ent[QN];         // cached router, adaptive policy: attention entropy per query
  double vsum[NW];
};

// Route + correct one (sequence, kv head) `bh` with the NW warps of the
// calling CTA.  `sm` is the CTA's scratch; the scores live in `dyn` when
// scores_in_smem, else in the workspace.  Every thread of the CTA calls it.
template <int QN, int NW, bool PF>
__device__ __forceinline__ void route_body(const DecodeArgs& a, int bh, RouteSmem<QN, NW>& sm, float* dyn,
                                           int scores_in_smem) {
  constexpr int NT = NW * 32;
  const Dims d = make_dims(a.cfg);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // prefill-correction inputs (PF): compiled out of the decode instantiation
  const float* const A_in = PF ? a.attn : nullptr;
  const float* const v_rows = PF ? a.v_rows : nullptr;
  const float* const v_pnorm = PF ? a.v_pnorm : nullptr;
  const float* const o_exact = PF ? a.o_exact : nullptr;
  const bool po_direct = PF && a.n_splits == 0;
  const int s = bh / d.H, h = bh % d.H;
  const int b = PF && a.seq_fixed >= 0 ? a.seq_fixed : a.seq_begin + s;
  const int D = d.D;
  const int Hq = a.act_heads;   // query heads per activation row
  // this CTA's query heads: q0 .. q0 + QN - 1 of the kv head's group of QG
  // (decode splits a group over gridDim.y CTAs, one query head each; the
  // prefill correction keeps the group in one CTA)
  const int QG = PF ? QN : QN * static_cast<int>(gridDim.y);
  const int q0 = PF ? 0 : QN * static_cast<int>(blockIdx.y);
  const int64_t lhp = d.lhp(b, a.layer, h);
  const int np = min(a.cache.num_pages[lhp], a.p_used);
  const carekv_route_params_t& rp = a.rp;

  // ── 1. queries and the merged split-K partials ──
  for (int idx = tid; idx < QN * D; idx += NT) {
    const int i = idx / D, c = idx % D;
    sm.Q[i][c] = load_act(a.q, (static_cast<int64_t>(s) * Hq + h * QG + q0 + i) * D + c, a.dt);
  }
  // every (query, channel) thread loads all splits' m, l and its O entry at
  // once (one round trip) and merges them; channel 0 publishes M, L
  if (tid == 0) { sm.cnt_k = 0; sm.cnt_v = 0; sm.ntot = 0; sm.any_k = 0; }
  for (int idx = tid; idx < QN * D; idx += NT) {
    const int i = idx / D, c = idx % D;
    const int64_t base = static_cast<int64_t>(bh) * a.n_splits * QG + q0 + i;
    if (po_direct) {   // po holds the base output itself, pm the logit row maxima (prefill)
      sm.O[i][c] = a.po[(static_cast<int64_t>(bh) * QG + q0 + i) * D + c];
      if (c == 0) {
        sm.M[i] = a.pm ? a.pm[static_cast<int64_t>(bh) * QG + q0 + i] : 0.f;
        sm.L[i] = 1.f;
        sm.invL[i] = 1.f;
        sm.mlb[i] = 0.f;
      }
      continue;
    }
    float M = -INFINITY;
    for (int sp = 0; sp < a.n_splits; ++sp) M = fmaxf(M, a.pm[base + sp * QG]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
      for (int sp = 0; sp < a.n_splits; ++sp) {
        const float m = a.pm[base + sp * QG];
        if (m == -INFINITY) continue;
        const float f = rex2((m - M) * kRL2e);
        L += a.pl[base + sp * QG] * f;
        O += a.po[(base + sp * QG) * D + c] * f;
      }
      O = __fdiv_rn(O, L);
    }
    sm.O[i][c] = O;
    if (c == 0) {
      sm.M[i] = M;
      sm.L[i] = L;
      sm.invL[i] = L > 0.f ? 1.0f / L : 0.f;
      sm.mlb[i] = L > 0.f ? fmaf(M, kRL2e, __log2f(L)) : INFINITY;
    }
  }
  __syncthreads();

  // attention weight of a logit of query i (the weight itself when a.S holds A)
  auto attw = [&](float sv, int i) -> float { return A_in ? sv : rex2((sv - sm.M[i]) * kRL2e) * sm.invL[i]; };

  // A fragments for the slot dots: rows gid = q_hi, gid+8 = q_lo of query gid;
  // k-step ks of group g covers channels g*32 + 8*tig + 4*ks + {0..3}
  const int nqfrag = a.kw != nullptr ? 0 : d.C * 2 * 32;   // unused when q.R_K is precomputed
  for (int x = tid; x < nqfrag; x += NT) {
    const int g = x / 64, ks = (x / 32) % 2, ln = x % 32;
    const int qg = ln >> 2, tg = ln & 3;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (qg < QN)
      for (int e = 0; e < 4; ++e) v[e] = sm.Q[qg][g * 32 + 8 * tg + 4 * ks + e];
    float hi[4], lo[4];
    for (int e = 0; e < 4; ++e) { hi[e] = __half2float(__float2half_rn(v[e])); lo[e] = v[e] - hi[e]; }
    sm.qfrag[g][ks][ln][0] = pack_h2(hi[0], hi[1]);
    sm.qfrag[g][ks][ln][1] = pack_h2(lo[0], lo[1]);
    sm.qfrag[g][ks][ln][2] = pack_h2(hi[2], hi[3]);
    sm.qfrag[g][ks][ln][3] = pack_h2(lo[2], lo[3]);
  }
  __syncthreads();

  auto write_base = [&]() {
    if (tid < QN) a.sel_out[(static_cast<int64_t>(bh) * QG + q0 + tid) * a.sel_stride] = 0;
    for (int idx = tid; idx < QN * D; idx += NT) {
      const int i = idx / D, c = idx % D;
      store_act(a.out, (static_cast<int64_t>(s) * Hq + h * QG + q0 + i) * D + c, sm.O[i][c], a.dt);
    }
  };
  if (np == 0 || rp.kind == CAREKV_KIND_NONE) {
    write_base();
    return;
  }

  const int KG = a.p_used * d.SK;
  const int VG = a.p_used * d.SV;
  const int NG = KG + VG;
  float* sc = scores_in_smem ? dyn : a.scores + (static_cast<int64_t>(bh) * QG + q0) * NG;
  const float* Sb = a.S + (static_cast<int64_t>(bh) * QG + q0) * a.p_used * kPage;
  // weights source: A itself when given (read through attw), else the logits
  const float* Wb = A_in ? A_in + (static_cast<int64_t>(bh) * QG + q0) * a.p_used * kPage : Sb;
  const int64_t sst = static_cast<int64_t>(a.p_used) * kPage;
  const bool kind_k = rp.kind == CAREKV_KIND_BOTH || rp.kind == CAREKV_KIND_K;
  const bool kind_v = rp.kind == CAREKV_KIND_BOTH || rp.kind == CAREKV_KIND_V;
  const bool may_k = kind_k && (rp.budget_mode == 0 ? rp.read_k > 0 : rp.ratio_k > 0.0);
  const bool may_v = kind_v && (rp.budget_mode == 0 ? rp.read_v > 0 : rp.ratio_v > 0.0);

  // ── 2a. K scores ──
  if (a.kw != nullptr) {
    // Thread per page: combined_kvscore of its stored K slots from q . R_K
    // precomputed by the split-K pass (||dS * A(1-A)|| over the page's valid
    // tokens * ||V_page||_F * sens), its V slots' block mass * error * sens,
    // and the slot / token counts -- all loads of a page in one round trip.
    int cntk = 0, cntv = 0, ntok = 0;
    for (int p = tid; p < a.p_used; p += NT) {
      const bool live = p < np;
      const int64_t pg = lhp * d.P + p;
      // every load of the page is issued before any result is used (the
      // workspace rows exist for every page, so no load waits on a check)
      const int nv = live ? a.cache.valid[pg] : 0;
      const float vc = live ? (v_pnorm ? v_pnorm[h * a.p_used + p] : sqrtf(a.cache.v_norm2[pg])) : 0.f;
      // the page's 4 V block errors in one load (NV == 4), so the error of a
      // kept block does not wait for the block index
      uint2 ve4 = make_uint2(0u, 0u);
      if (live && d.NV == 4) ve4 = *reinterpret_cast<const uint2*>(a.cache.v_err + pg * 4);
      // the first V slot's block, loaded before any score store (the scores
      // may live in global memory, and a later load would wait for them)
      const int vb0 = live && d.SV > 0 ? a.cache.v_slot_block[pg * d.SV] : -1;
      ntok += nv;
      for (int i = 0; i < QN; ++i) {
        const float4* srow = reinterpret_cast<const float4*>(Wb + i * sst + p * kPage);
        float sv[16];
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const float4 x = srow[q4];
          sv[4 * q4] = x.x; sv[4 * q4 + 1] = x.y; sv[4 * q4 + 2] = x.z; sv[4 * q4 + 3] = x.w;
        }
        // attention weight of position j (token pos_tok(j)); 0 past the valid
        // rows: 2^(s log2(e) - M log2(e) - log2(L))
        float A[16];
        const float mlb = sm.mlb[i];
#pragma unroll
        for (int j = 0; j < 16; ++j)
          A[j] = pos_tok(j, a.s_perm) < nv ? (A_in ? sv[j] : rex2(fmaf(sv[j], kRL2e, -mlb))) : 0.f;
        // attention mass of each 4-token V block (positions in ascending order)
        float bm[4] = {0.f, 0.f, 0.f, 0.f};
        if (d.vtb == 4) {
          if (a.s_perm) {
#pragma unroll
            for (int j = 0; j < 16; ++j) bm[((j >> 1) + 8 * (j & 1)) >> 2] += A[j];
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) bm[j >> 2] += A[j];
          }
        }
        for (int j = 0; j < d.SK; ++j) {
          const int e = p * d.SK + j;
          const int grp = live ? a.cache.k_slot_group[pg * d.SK + j] : -1;
          const float4* wrow = reinterpret_cast<const float4*>(a.kw + ((static_cast<int64_t>(bh) * QG + q0 + i) * KG + e) * kPage);
          // ||dS * A(1-A)|| with dS = q.R_K / sqrt(D): the 1/sqrt(D) is
          // applied to the root
          float ss = 0.f;
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const float4 w4 = wrow[q4];
            const float wa[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float Au = A[4 * q4 + u];
              const float term = wa[u] * fmaf(-Au, Au, Au);
              ss = fmaf(term, term, ss);
            }
          }
          const bool ok = grp >= 0 && nv > 0;
          if (i == 0) cntk += ok;
          float v = -1.f;
          if (ok && may_k) {
            float ks = sqrtf(ss) * a.sf * vc;
            if (!(ks == ks) || isinf(ks)) ks = 0.f;
            v = fmaxf(ks, 0.f) * rp.sensitivity;
          }
          sc[i * NG + e] = v;
        }
        for (int j = 0; j < d.SV; ++j) {
          const int e = p * d.SV + j;
          const int vb = live ? (j == 0 ? vb0 : a.cache.v_slot_block[pg * d.SV + j]) : -1;
          const int t0 = vb * d.vtb, t1 = min(t0 + d.vtb, nv);
          const bool ok = vb >= 0 && t1 > t0;
          if (i == 0) cntv += ok;
          float v = -1.f;
          if (ok && may_v) {
            const float err = f16_bits_to_f32(d.NV == 4 ? static_cast<uint16_t>(((vb & 2) ? ve4.y : ve4.x) >> (16 * (vb & 1)))
                                                        : a.cache.v_err[pg * d.NV + vb]);
            float mass = 0.f;
            if (d.vtb == 4) {
              mass = vb == 0 ? bm[0] : (vb == 1 ? bm[1] : (vb == 2 ? bm[2] : bm[3]));
            } else {
#pragma unroll
              for (int jj = 0; jj < 16; ++jj) {
                const int t = pos_tok(jj, a.s_perm);
                if (t >= t0 && t < t1) mass += A[jj];
              }
            }
            v = __fmul_rn(__fmul_rn(mass, err), rp.sensitivity);
          }
          sc[i * NG + KG + e] = v;
        }
      }
    }
    cntk = __reduce_add_sync(0xffffffffu, cntk);
    cntv = __reduce_add_sync(0xffffffffu, cntv);
    ntok = __reduce_add_sync(0xffffffffu, ntok);
    if (lane == 0) {
      if (cntk) atomicAdd(&sm.cnt_k, cntk);
      if (cntv) atomicAdd(&sm.cnt_v, cntv);
      if (ntok) atomicAdd(&sm.ntot, ntok);
    }
  } else if (rp.kscore_live || !may_k) {
    // combined_kvscore, one warp per stored slot: q . R_K^T on the tensor
    // cores (codes as exact fp16 integers, slot scale applied after), then
    // ||dS * A(1-A)|| over the page's valid tokens * ||V_page||_F * sens.
    const int gid = lane >> 2, tig = lane & 3;
    int cnt = 0;
    // Every load of a slot is issued at once: the arena rows exist for every
    // page below max_pages, so none waits on the slot's group or the page's
    // count.
    struct SlotLd {
      int grp, nv;
      uint32_t w0, w1;
      uint16_t rs;
      float vn, s4[4];
    };
    auto slot_load = [&](int e, SlotLd& x) {
      const int p = e / d.SK, j = e % d.SK;
      const int64_t pg = lhp * d.P + p;
      const bool live = e < KG && p < np;
      const int64_t si = live ? pg * d.SK + j : 0;
      const int64_t pgl = live ? pg : 0;
      x.grp = live ? a.cache.k_slot_group[si] : -1;
      x.nv = live ? a.cache.valid[pgl] : 0;
      const uint8_t* pay = a.cache.k_slot_data + si * d.kslot_bytes;
      x.w0 = *reinterpret_cast<const uint32_t*>(pay + gid * 16 + 4 * tig);
      x.w1 = *reinterpret_cast<const uint32_t*>(pay + (gid + 8) * 16 + 4 * tig);
      x.rs = a.cache.k_slot_scale[si];
      x.vn = v_pnorm ? (live ? v_pnorm[h * a.p_used + p] : 0.f) : a.cache.v_norm2[pgl];
#pragma unroll
      for (int u = 0; u < 4; ++u) x.s4[u] = 0.f;
      if (gid < QN && live) {
        const float* srow = Wb + gid * sst + p * kPage;
        x.s4[0] = srow[tok_pos(2 * tig, a.s_perm)];
        x.s4[1] = srow[tok_pos(2 * tig + 1, a.s_perm)];
        x.s4[2] = srow[tok_pos(8 + 2 * tig, a.s_perm)];
        x.s4[3] = srow[tok_pos(9 + 2 * tig, a.s_perm)];
      }
    };
    for (int e = warp; e < KG; e += NW) {
      SlotLd cur;
      slot_load(e, cur);
      const int grp = cur.grp, nv = cur.nv;
      const bool ok = grp >= 0 && nv > 0;
      cnt += ok;
      if (!ok || !may_k) {
        if (lane < QN) sc[lane * NG + e] = -1.f;
        continue;
      }
      const uint32_t w0 = cur.w0, w1 = cur.w1;
      const float rs = f16_bits_to_f32(cur.rs);
      const float vc = v_pnorm ? cur.vn : sqrtf(cur.vn);
      const float s4[4] = {cur.s4[0], cur.s4[1], cur.s4[2], cur.s4[3]};
      float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) {
        const uint4 af = *reinterpret_cast<const uint4*>(&sm.qfrag[grp][ks][lane][0]);
        mma_f16(c0, af.x, af.y, af.z, af.w, nib_pair(w0, 2 * ks), nib_pair(w0, 2 * ks + 1));
        mma_f16(c1, af.x, af.y, af.z, af.w, nib_pair(w1, 2 * ks), nib_pair(w1, 2 * ks + 1));
      }
      // tokens 2tig, 2tig+1 (c0) and 8+2tig, 9+2tig (c1) of query gid
      float ss = 0.f;
      if (gid < QN) {
        const float dots[4] = {c0[0] + c0[2], c0[1] + c0[3], c1[0] + c1[2], c1[1] + c1[3]};
        const int toks[4] = {2 * tig, 2 * tig + 1, 8 + 2 * tig, 9 + 2 * tig};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (toks[u] < nv) {
            const float dS = __fdiv_rn(__fmul_rn(dots[u], rs), a.sqrt_d);
            const float A = attw(s4[u], gid);
            const float term = dS * (A * (1.f - A));
            ss = fmaf(term, term, ss);
          }
        }
      }
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      ss += __shfl_xor_sync(0xffffffffu, ss, 2);
      if (tig == 0 && gid < QN) {
        float ks = sqrtf(ss) * vc;
        if (!(ks == ks) || isinf(ks)) ks = 0.f;
        sc[gid * NG + e] = fmaxf(ks, 0.f) * rp.sensitivity;
      }
    }
    if (lane == 0 && cnt) atomicAdd(&sm.cnt_k, cnt);
  } else
  {
    const int half = lane >> 4, t = lane & 15;
    const unsigned hm = 0xFFFFu << (16 * half);   // shuffles stay inside the half-warp
    int cnt = 0;
    for (int e0 = 2 * warp; e0 < KG; e0 += 2 * NW) {
      const int e = e0 + half;
      const bool in = e < KG;
      const int p = in ? e / d.SK : 0;
      const int j = in ? e % d.SK : 0;
      const int64_t pg = lhp * d.P + p;
      int grp = -1, nv = 0;
      if (in && p < np) {
        grp = a.cache.k_slot_group[pg * d.SK + j];
        nv = a.cache.valid[pg];
      }
      const bool ok = grp >= 0 && nv > 0;
      if (t == 0 && ok) ++cnt;
      if (!ok || !may_k) {
        if (in && t < QN) sc[t * NG + e] = -1.f;
        continue;
      }
      const uint8_t* pay = a.cache.k_slot_data + (pg * d.SK + j) * d.kslot_bytes;
      const uint4 raw = *reinterpret_cast<const uint4*>(pay + t * 16);
      const float rs = f16_bits_to_f32(a.cache.k_slot_scale[pg * d.SK + j]);
      float sv[QN], wv[QN];   // logits and attention weights
#pragma unroll
      for (int i = 0; i < QN; ++i) {
        sv[i] = t < nv && a.S ? Sb[i * sst + p * kPage + tok_pos(t, a.s_perm)] : 0.f;
        wv[i] = t < nv ? (A_in ? Wb[i * sst + p * kPage + tok_pos(t, a.s_perm)] : attw(sv[i], i)) : 0.f;
      }
      const float vn2 = v_pnorm ? v_pnorm[h * a.p_used + p] * v_pnorm[h * a.p_used + p] : a.cache.v_norm2[pg];
      const uint32_t wds[4] = {raw.x, raw.y, raw.z, raw.w};
      float r[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        int v = (wds[c >> 3] >> (4 * (c & 7))) & 15;
        v = v > 7 ? v - 16 : v;
        r[c] = __fmul_rn(static_cast<float>(v), rs);
      }
      const float* qb = &sm.Q[0][grp * d.kcg];
      if (rp.kscore_live) {
        const float vc = sqrtf(vn2);
#pragma unroll
        for (int i = 0; i < QN; ++i) {
          float dot = 0.f;
#pragma unroll
          for (int c = 0; c < 32; ++c) dot = fmaf(qb[i * 128 + c], r[c], dot);
          float term = 0.f;
          if (t < nv) {
            const float dS = __fdiv_rn(dot, a.sqrt_d);
            const float A = wv[i];
            term = dS * (A * (1.f - A));
          }
          float ss = term * term;
          ss += __shfl_xor_sync(hm, ss, 8);
          ss += __shfl_xor_sync(hm, ss, 4);
          ss += __shfl_xor_sync(hm, ss, 2);
          ss += __shfl_xor_sync(hm, ss, 1);
          float ks = sqrtf(ss) * vc;
          if (!(ks == ks) || isinf(ks)) ks = 0.f;
          if (t == 0) sc[i * NG + e] = fmaxf(ks, 0.f) * rp.sensitivity;
        }
      } else {
        // sketch proxy: mass * |q_sketch . k_sketch| * boundary * vdiff * sens
        const float mv = d.scale_mode == CAREKV_SCALE_INT8 ? f16_bits_to_f32(a.cache.v_master[pg]) : 0.f;
        for (int i = 0; i < QN; ++i) {
          float A = 0.f, inv = 0.f, vd = 0.f;
          if (t < nv) {
            A = wv[i];
            inv = __fdiv_rn(1.f, fmaxf(sm.M[i] - sv[i], kREps));
            float acc = 0.f;
            for (int c = 0; c < D; ++c) {
              float vh;
              if (v_rows) {
                vh = v_rows[((static_cast<int64_t>(h) * a.p_used + p) * kPage + t) * D + c];
              } else {
                const int64_t si = (pg * kPage + t) * d.G + c / d.gsize;
                const float svv = d.kivi ? reinterpret_cast<const float*>(a.cache.v_scale)[si]
                                         : read_scale(a.cache.v_scale, si, d.scale_mode, mv);
                const int cv = unpack_code(a.cache.v_codes + (pg * kPage + t) * d.R, c, d.bits);
                vh = d.kivi ? f16r(kivi_hat(cv, svv, a.dt)) : f16r(__fmul_rn(static_cast<float>(cv), svv));
              }
              const float df = vh - sm.O[i][c];
              acc = fmaf(df, df, acc);
            }
            vd = sqrtf(acc);
          }
          float mass = A, bnd = A * inv, pvd = A * vd;
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) {
            mass += __shfl_xor_sync(hm, mass, o);
            bnd += __shfl_xor_sync(hm, bnd, o);
            pvd += __shfl_xor_sync(hm, pvd, o);
          }
          float qd = 0.f;
          for (int jj = t; jj < d.sketch; jj += 16) {
            float qs = 0.f;
            for (int c = 0; c < d.kcg; ++c) qs = fmaf(sm.Q[i][grp * d.kcg + c], a.sketch_proj[c * d.sketch + jj], qs);
            qd += qs * f16_bits_to_f32(a.cache.k_sketch[(pg * d.C + grp) * d.sketch + jj]);
          }
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) qd += __shfl_xor_sync(hm, qd, o);
          if (t == 0) {
            // residual_router.py:185-212 (the cached router's baseline_score
            // ablations; the vectorized proxy is the "carekv" score)
            float v;
            switch (rp.legacy ? rp.baseline_score : CAREKV_SCORE_CAREKV) {
              case CAREKV_SCORE_MAGNITUDE_ONLY: v = fabsf(qd); break;
              case CAREKV_SCORE_ATTENTION_ONLY: v = mass; break;
              case CAREKV_SCORE_ORACLE_PROXY: v = fabsf(qd) * mass; break;
              default: v = mass * fabsf(qd) * bnd * pvd * rp.sensitivity;
            }
            sc[i * NG + e] = v;
          }
        }
      }
    }
    cnt += __shfl_xor_sync(0xffffffffu, cnt, 16);
    if (lane == 0 && cnt) atomicAdd(&sm.cnt_k, cnt);
  }
  // ── 2b. V scores: thread per grid entry; page token count ──
  if (a.kw == nullptr) {
    int cnt = 0, ntok = 0;
    for (int e = tid; e < VG; e += NT) {
      const int p = e / d.SV, j = e % d.SV;
      const int64_t pg = lhp * d.P + p;
      int vb = -1, nv = 0;
      if (p < np) {
        vb = a.cache.v_slot_block[pg * d.SV + j];
        nv = a.cache.valid[pg];
      }
      const int t0 = vb * d.vtb, t1 = min(t0 + d.vtb, nv);
      const bool ok = vb >= 0 && t1 > t0;
      cnt += ok;
      if (ok && may_v) {
        const float err = f16_bits_to_f32(a.cache.v_err[pg * d.NV + vb]);
        for (int i = 0; i < QN; ++i) {
          float mass = 0.f;
          for (int t = t0; t < t1; ++t)
            mass += attw(Wb[i * sst + p * kPage + tok_pos(t, a.s_perm)], i);
          float v;
          switch (rp.legacy ? rp.baseline_score : CAREKV_SCORE_CAREKV) {
            case CAREKV_SCORE_MAGNITUDE_ONLY: v = err; break;
            case CAREKV_SCORE_ATTENTION_ONLY: v = mass; break;
            case CAREKV_SCORE_ORACLE_PROXY: v = __fmul_rn(mass, err); break;
            default: v = __fmul_rn(__fmul_rn(mass, err), rp.sensitivity);
          }
          sc[i * NG + KG + e] = v;
        }
      } else {
        for (int i = 0; i < QN; ++i) sc[i * NG + KG + e] = -1.f;
      }
    }
    for (int p = tid; p < np; p += NT) ntok += a.cache.valid[lhp * d.P + p];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
      ntok += __shfl_xor_sync(0xffffffffu, ntok, o);
    }
    if (lane == 0) {
      if (cnt) atomicAdd(&sm.cnt_v, cnt);
      if (ntok) atomicAdd(&sm.ntot, ntok);
    }
  }
  __syncthreads();

  // ── budgets (residual_router.py:37-76) ──
  const int n_k = sm.cnt_k, n_v = sm.cnt_v, ntot_all = sm.ntot;
  const bool want_k = kind_k && n_k > 0, want_v = kind_v && n_v > 0;
  int bk, bv;
  {
    const int tk = want_k ? n_k : 0, tv = want_v ? n_v : 0;
    if (rp.budget_mode == 0) {
      bk = rp.read_k;
      bv = rp.read_v;
    } else {
      bk = (rp.ratio_k > 0.0 && tk > 0) ? max(1, static_cast<int>(static_cast<double>(tk) * rp.ratio_k)) : 0;
      bv = (rp.ratio_v > 0.0 && tv > 0) ? max(1, static_cast<int>(static_cast<double>(tv) * rp.ratio_v)) : 0;
    }
    if (rp.kind == CAREKV_KIND_V) bk = 0;
    if (rp.kind == CAREKV_KIND_K) bv = 0;
    bk = min(bk, tk);
    bv = min(bv, tv);
  }
  if ((!want_k && !want_v) || (bk == 0 && bv == 0)) {
    write_base();
    return;
  }
  const bool score_k = want_k && bk > 0, score_v = want_v && bv > 0;

  // ── 3a. normalisation; kinds that take no part are not candidates ──
  // the cached router normalises whenever kind is "both" and ranks every
  // candidate of an enabled kind (residual_router.py:318-348); the
  // vectorized router only kinds with a budget
  const bool norm = rp.legacy ? (rp.score_normalize && rp.kind == CAREKV_KIND_BOTH)
                              : (rp.score_normalize && rp.kind == CAREKV_KIND_BOTH && score_k && score_v);
  if (norm) {
    for (int i = 0; i < QN; ++i) {
      float ak = 0.f, av = 0.f;
      for (int e = tid; e < NG; e += NT) {
        const float v = sc[i * NG + e];
        if (v >= 0.f) { if (e < KG) ak += v; else av += v; }
      }
      ak = warp_sum(ak);
      av = warp_sum(av);
      if (lane == 0) { sm.red[warp][i] = ak; sm.red2[warp][i] = av; }
    }
    __syncthreads();
    if (tid < QN) {
      float x = 0.f, y = 0.f;
      for (int w = 0; w < NW; ++w) { x += sm.red[w][tid]; y += sm.red2[w][tid]; }
      sm.nk[tid] = fmaxf(__fdiv_rn(x, static_cast<float>(n_k)), kREps);
      sm.nv[tid] = fmaxf(__fdiv_rn(y, static_cast<float>(n_v)), kREps);
    }
    __syncthreads();
  }
  for (int e = tid; e < NG; e += NT) {
    const bool part = rp.legacy ? (e < KG ? want_k : want_v) : (e < KG ? score_k : score_v);
    for (int i = 0; i < QN; ++i) {
      float v = sc[i * NG + e];
      if (!part) v = -1.f;
      else if (norm && v >= 0.f) {
        v = e < KG ? __fdiv_rn(v, sm.nk[i]) : __fdiv_rn(v, sm.nv[i]);
        if (rp.kscore_live) v = __fmul_rn(v, e < KG ? rp.lambda_k : rp.lambda_v);
      }
      sc[i * NG + e] = v;
    }
  }
  __syncthreads();

  // ── 3b. selection ──
  const bool joint = rp.joint && rp.kind == CAREKV_KIND_BOTH && score_k && score_v;
  // Top-k of sc[i][lo:hi) by (score desc, index asc), appended to sel[i].
  // Every warp keeps a running top-32 of its 64-entry blocks (bitonic sort
  // of the block on the warp's shuffles, then a bitonic merge with the
  // running list); warp 0 merges the warps' lists the same way.  Excluded
  // entries hold a negative score and sort last.
  // Publish the first n of a sorted list (one element per lane) into sel[i].
  int* const gsel_base = a.sel_out + (static_cast<int64_t>(bh) * QG + q0) * a.sel_stride;
  auto publish = [&](int i, float mv, int mi, int k) {
    const int base = sm.nsel[i];
    int n = __popc(__ballot_sync(0xffffffffu, mv >= 0.f));
    n = min(n, k);
    if (lane < n) {
      gsel_base[i * a.sel_stride + 1 + base + lane] = mi;
      if (base + lane < kRSel) sm.sel[i][base + lane] = mi;
    }
    if (__any_sync(0xffffffffu, lane < n && mi < KG) && lane == 0) sm.any_k = 1;
    __syncwarp();
    if (lane == 0) sm.nsel[i] = base + n;
  };
  // exclusive prefix sum of v over the CTA's threads (thread order); every
  // thread calls it
  auto block_scan = [&](int v, int& total) -> int {
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) sm.scan[warp] = x;
    __syncthreads();
    int before = 0;
    total = 0;
    for (int w = 0; w < NW; ++w) {
      const int t = sm.scan[w];
      if (w < warp) before += t;
      total += t;
    }
    __syncthreads();
    return before + x - v;
  };
  // Top-k (k > kRSel) of sc[i][lo:hi) by (score desc, index asc), appended
  // to the selection in index order.  Radix select on the candidates'
  // score bits (non-negative fp32 scores order like their bit patterns),
  // four 8-bit digits from the top, finds the k-th score T; every entry
  // above T is taken and, of the entries equal to T, the lowest indices
  // (a block-wide stable compaction in index order).
  auto pick_large = [&](int i, int lo, int hi, int k) {
    const float* row = sc + i * NG;
    auto key_of = [&](int e, bool& cand) -> uint32_t {
      const float x = row[e];
      cand = x >= 0.f;   // NaN and excluded entries (negative) are not candidates
      return __float_as_uint(__fadd_rn(x, 0.0f));
    };
    int ncand = 0;
    for (int e = lo + tid; e < hi; e += NT) {
      bool c;
      (void)key_of(e, c);
      ncand += c;
    }
    int tot = 0;
    (void)block_scan(ncand, tot);
    const int need = min(k, tot);
    if (need <= 0) return;
    uint32_t prefix = 0, pmask = 0;
    int remaining = need;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int x = tid; x < 256; x += NT) sm.hist[x] = 0;
      __syncthreads();
      for (int e = lo + tid; e < hi; e += NT) {
        bool c;
        const uint32_t u = key_of(e, c);
        if (c && (u & pmask) == prefix) atomicAdd(&sm.hist[(u >> shift) & 255], 1);
      }
      __syncthreads();
      if (warp == 0) {
        // lane l holds digits 255-8l .. 248-8l (descending); suffix counts
        int cnt[8], own = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) { cnt[j] = sm.hist[255 - 8 * lane - j]; own += cnt[j]; }
        int incl = own;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        const int above = incl - own;   // entries in digits above this lane's range
        // the lane whose range holds the remaining-th largest entry
        const bool mine = above < remaining && remaining <= incl;
        if (mine) {
          int acc = above;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if (acc + cnt[j] >= remaining) {
              sm.rsel[0] = 255 - 8 * lane - j;
              sm.rsel[1] = remaining - acc;
              break;
            }
            acc += cnt[j];
          }
        }
      }
      __syncthreads();
      prefix |= static_cast<uint32_t>(sm.rsel[0]) << shift;
      pmask |= 255u << shift;
      remaining = sm.rsel[1];
      __syncthreads();
    }
    // prefix = T (exact score bits); remaining = entries equal to T to take
    const int len = hi - lo, chunk = (len + NT - 1) / NT;
    const int c0 = lo + min(len, tid * chunk), c1 = lo + min(len, (tid + 1) * chunk);
    int gt = 0, eq = 0;
    for (int e = c0; e < c1; ++e) {
      bool c;
      const uint32_t u = key_of(e, c);
      if (c) { gt += u > prefix; eq += u == prefix; }
    }
    int t2 = 0;
    const int eq_before = block_scan(eq, t2);
    const int take = max(0, min(eq, remaining - eq_before));
    const int off = block_scan(gt + take, t2);
    const int base = sm.nsel[i];
    int* g = gsel_base + i * a.sel_stride + 1 + base + off;
    int w = 0, te = 0;
    bool anyk = false;
    for (int e = c0; e < c1; ++e) {
      bool c;
      const uint32_t u = key_of(e, c);
      const bool tk = c && (u > prefix || (u == prefix && te++ < take));
      if (tk) {
        g[w] = e;
        if (base + off + w < kRSel) sm.sel[i][base + off + w] = e;
        ++w;
        anyk |= e < KG;
      }
    }
    if (anyk) sm.any_k = 1;
    __syncthreads();
    if (tid == 0) sm.nsel[i] = base + t2;
    __syncthreads();
  };
  auto pick = [&](int i, int lo, int hi, int k) {
    if (k <= 0 || hi <= lo) return;
    if (k > kRSel) {
      pick_large(i, lo, hi, k);
      return;
    }
    const float* row = sc + i * NG;
    // ── prefilter: tau = min over warps of each warp's r-th best lane
    // maximum, r = ceil(k / NW); the r best lanes of every warp hold
    // distinct entries >= tau, so at least NW*r >= k entries score >= tau
    // and the top-k are among them.  With <= 64 such entries one warp sorts
    // them; else (ties, or warps with fewer than r live lanes) the full path
    // runs.
    {
      const int r = (k + NW - 1) / NW;   // <= kRSel / NW <= 32
      // r-th best lane maximum of the warp: each lane's best entry, then a
      // descending bitonic sort of the 32 lane maxima (values only)
      float lv = -2.f;
      for (int e = lo + tid; e < hi; e += NT) {
        const float x = row[e];
        lv = fmaxf(lv, x == x ? x : -1.f);
      }
#pragma unroll
      for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
          const float o = __shfl_xor_sync(0xffffffffu, lv, stride);
          lv = (((lane & stride) == 0) == ((lane & size) == 0)) ? fmaxf(lv, o) : fminf(lv, o);
        }
      }
      lv = __shfl_sync(0xffffffffu, lv, r - 1);
      if (lane == 0) sm.gv[warp] = lv;
      if (tid == 0) sm.gcount = 0;
      __syncthreads();
      float tau = sm.gv[0];
      for (int w = 1; w < NW; ++w) tau = fminf(tau, sm.gv[w]);
      if (tau >= 0.f) {
        // candidates: one slot reservation per warp and pass (ballot), -0
        // folded onto +0 so that float order is the key order
        for (int e0 = lo; e0 < hi; e0 += NT) {
          const int e = e0 + tid;
          const float x = e < hi ? row[e] : -1.f;
          const bool c = x >= tau;
          const unsigned bc = __ballot_sync(0xffffffffu, c);
          int slot0 = 0;
          if (lane == 0 && bc) slot0 = atomicAdd(&sm.gcount, __popc(bc));
          slot0 = __shfl_sync(0xffffffffu, slot0, 0);
          const int slot = slot0 + __popc(bc & ((1u << lane) - 1u));
          if (c && slot < 64) {
            sm.gv[32 + slot] = __fadd_rn(x, 0.0f);
            sm.gi[32 + slot] = e;
          }
        }
        __syncthreads();
        const int nc = sm.gcount;
        if (nc <= 64) {
          // rank of every candidate under (score desc, index asc): the
          // candidates ahead of it; ranks below k are published in rank order
          // (all candidates score >= tau >= 0)
          const int base = sm.nsel[i];
          const int n = min(nc, k);
          if (tid < nc) {
            const float x = sm.gv[32 + tid];
            const int ix = sm.gi[32 + tid];
            int r = 0;
            for (int j = 0; j < nc; ++j) {
              const float y = sm.gv[32 + j];
              r += (y > x || (y == x && sm.gi[32 + j] < ix)) ? 1 : 0;
            }
            if (r < n) {
              gsel_base[i * a.sel_stride + 1 + base + r] = ix;
              if (base + r < kRSel) sm.sel[i][base + r] = ix;
              if (ix < KG) sm.any_k = 1;
            }
          }
          __syncthreads();
          if (tid == 0) sm.nsel[i] = base + n;
          __syncthreads();
          return;
        }
      }
      __syncthreads();
    }
    uint64_t run = rkey(-2.f, 0x7fffffff);
    for (int b0 = lo + warp * 64; b0 < hi; b0 += NW * 64) {
      const int e0 = b0 + lane, e1 = b0 + lane + 32;
      float v0 = e0 < hi ? row[e0] : -2.f, v1 = e1 < hi ? row[e1] : -2.f;
      v0 = v0 == v0 ? v0 : -1.f;
      v1 = v1 == v1 ? v1 : -1.f;
      uint64_t k0 = rkey(v0, e0 < hi ? e0 : 0x7fffffff), k1 = rkey(v1, e1 < hi ? e1 : 0x7fffffff);
      rsort64(k0, k1, lane);
      run = rmerge32(run, k0, lane);
    }
    sm.gv[warp * 32 + lane] = rkey_score(run);
    sm.gi[warp * 32 + lane] = rkey_index(run);
    __syncthreads();
    if (warp == 0) {
      uint64_t m = rkey(sm.gv[lane], sm.gi[lane]);
      for (int w = 1; w < NW; ++w) m = rmerge32(m, rkey(sm.gv[w * 32 + lane], sm.gi[w * 32 + lane]), lane);
      publish(i, rkey_score(m), rkey_index(m), k);
    }
    __syncthreads();
  };
  if (tid < QN) sm.nsel[tid] = 0;
  __syncthreads();
  // cached router, adaptive policy: attention entropy of each query over
  // the valid tokens, -sum max(A, eps) log max(A, eps) (residual_router.py:369-376)
  if (rp.legacy && rp.policy == CAREKV_POLICY_ADAPTIVE) {
    for (int i = 0; i < QN; ++i) {
      float ent = 0.f;
      for (int x = tid; x < np * kPage; x += NT) {
        const int p = x >> 4, t = x & (kPage - 1);
        if (t < a.cache.valid[lhp * d.P + p]) {
          const float av = fmaxf(attw(Wb[i * sst + p * kPage + tok_pos(t, a.s_perm)], i), kREps);
          ent -= av * logf(av);
        }
      }
      ent = warp_sum(ent);
      if (lane == 0) sm.red[warp][i] = ent;
    }
    __syncthreads();
    if (tid < QN) {
      float e = 0.f;
      for (int w = 0; w < NW; ++w) e += sm.red[w][tid];
      sm.ent[tid] = e;
    }
    __syncthreads();
  }
  // Keep, of the selected entries of query i, those passing the
  // adaptive_score thresholds per kind: score >= rel * the kind's top score
  // and >= abs; a kind left with fewer than min_keep keeps its min_keep best
  // (residual_router.py:393-433).  At most 32 entries (host-checked).
  auto thresholds = [&](int i) {
    if (warp == 0) {
      const int n = sm.nsel[i];
      const int e = lane < n ? sm.sel[i][lane] : 0x7fffffff;
      const float sv = lane < n ? sc[i * NG + e] : -1.f;
      const bool isk = lane < n && e < KG, isv = lane < n && e >= KG;
      float topk = isk ? sv : -1.f, topv = isv ? sv : -1.f;
      topk = warp_max(topk);
      topv = warp_max(topv);
      const float top = isk ? topk : topv;
      const bool pass = (lane < n) && (rp.rel_threshold <= 0.f || sv >= rp.rel_threshold * top) &&
                        (rp.abs_threshold <= 0.f || sv >= rp.abs_threshold);
      int rank = 0;
      for (int j = 0; j < n; ++j) {
        const int ej = __shfl_sync(0xffffffffu, e, j);
        const float sj = __shfl_sync(0xffffffffu, sv, j);
        if ((ej < KG) == isk && (sj > sv || (sj == sv && ej < e))) ++rank;
      }
      const int npass = __popc(__ballot_sync(0xffffffffu, pass && isk)) * isk +
                        __popc(__ballot_sync(0xffffffffu, pass && isv)) * isv;
      const int nkind = __popc(__ballot_sync(0xffffffffu, isk)) * isk + __popc(__ballot_sync(0xffffffffu, isv)) * isv;
      const bool keep = (lane < n) && (rp.min_keep > 0 && npass < rp.min_keep ? rank < min(rp.min_keep, nkind) : pass);
      const unsigned km = __ballot_sync(0xffffffffu, keep);
      const int pos = __popc(km & ((1u << lane) - 1u));
      __syncwarp();
      if (keep) {
        sm.sel[i][pos] = e;
        gsel_base[i * a.sel_stride + 1 + pos] = e;
      }
      __syncwarp();
      if (lane == 0) sm.nsel[i] = __popc(km);
    }
    __syncthreads();
  };
  for (int i = 0; i < QN; ++i) {
    if (rp.legacy) {
      // ResidualRouter.route policies (residual_router.py:325-390)
      if (rp.policy == CAREKV_POLICY_JOINT) {
        const int mb = (bk > 0 && bv > 0) ? bk + bv : max(bk, bv);
        pick(i, 0, NG, min(mb, n_k + n_v));
      } else if (rp.policy == CAREKV_POLICY_K_FIRST) {
        pick(i, 0, KG, bk);
        const int rem = max(0, bk + bv - sm.nsel[i]);
        if (rem > 0 && n_v > 0) {
          // V candidates at or above the mean V score, best first
          double vs = 0.0;
          int vc = 0;
          for (int e = KG + tid; e < NG; e += NT) {
            const float v = sc[i * NG + e];
            if (v >= 0.f) { vs += v; ++vc; }
          }
          for (int o = 16; o > 0; o >>= 1) {
            vs += __shfl_xor_sync(0xffffffffu, vs, o);
            vc += __shfl_xor_sync(0xffffffffu, vc, o);
          }
          if (lane == 0) { sm.vsum[warp] = vs; sm.scan[warp] = vc; }
          __syncthreads();
          double tv = 0.0;
          int tc = 0;
          for (int w = 0; w < NW; ++w) { tv += sm.vsum[w]; tc += sm.scan[w]; }
          const double vmean = tc > 0 ? tv / tc : 0.0;
          __syncthreads();
          for (int e = KG + tid; e < NG; e += NT) {
            const float v = sc[i * NG + e];
            if (v >= 0.f && static_cast<double>(v) < vmean) sc[i * NG + e] = -1.f;
          }
          __syncthreads();
          pick(i, KG, NG, rem);
        }
      } else if (rp.policy == CAREKV_POLICY_ADAPTIVE) {
        const int tot = bk + bv;
        if (tot > 0) {
          const double vf = fmin(1.0, fmax(0.0, static_cast<double>(sm.ent[i]) / log(static_cast<double>(max(ntot_all, 2)))));
          const int va = max(0, static_cast<int>(rint(tot * vf)));   // Python round: half to even
          const int ka = max(0, tot - va);
          pick(i, 0, KG, ka);
          pick(i, KG, NG, va);
        }
      } else {
        pick(i, 0, KG, bk);
        pick(i, KG, NG, bv);
      }
      if (rp.adaptive_score) thresholds(i);
    } else if (joint) {
      const int mb = (bk > 0 && bv > 0) ? bk + bv : max(bk, bv);
      pick(i, 0, NG, min(mb, n_k + n_v));
    } else {
      if (score_k) pick(i, 0, KG, bk);
      if (score_v) pick(i, KG, NG, bv);
    }
  }
  if (tid < QN) gsel_base[tid * a.sel_stride] = sm.nsel[tid];
  if (scores_in_smem) {
    float* g = a.scores + (static_cast<int64_t>(bh) * QG + q0) * NG;
    for (int e = tid; e < QN * NG; e += NT) g[e] = sc[e];
  }
  __syncthreads();

  // ── 4. apply ──
  const bool exact = rp.exact && sm.any_k;
  const int ntot = sm.ntot;
  int reads_k = 0, reads_v = 0;
  const int R = d.R, G = d.G;
  // INT3 rows with int8 scales decode a packed word (8 channels) per lane;
  // other layouts decode channel by channel
  const bool fast3 = d.bits == 3 && d.scale_mode == CAREKV_SCALE_INT8 && (D == 64 || D == 128) && d.gsize % 8 == 0;
  const int WPR = D / 8;      // packed words (8 channels) per row
  const int RG = 32 / WPR;    // rows one warp walks side by side
  const int wl = lane % WPR, rg = lane / WPR;
  // Staging of the selected items (a K page: its packed V rows, V scales and
  // logits; a V slot: its payload and its page's logits) in batches that fit
  // sm.stg.  Every segment is a multiple of 16 bytes; with 16-byte aligned
  // sources the lanes of warp 0 stage a batch with bulk copies (one round
  // trip), else every warp copies its own items.
  const int es = d.scale_mode == CAREKV_SCALE_INT8 ? 1 : (d.scale_mode == CAREKV_SCALE_F32 ? 4 : 2);
  const int k_codes_b = kPage * R, k_sc_b = kPage * G * es;
  const int k_item_b = k_codes_b + k_sc_b + kPage * 4;
  const int v_item_b = d.vslot_bytes + kPage * 4;
  const bool bulk = ((reinterpret_cast<uintptr_t>(a.cache.v_codes) | reinterpret_cast<uintptr_t>(a.cache.v_scale) |
                      reinterpret_cast<uintptr_t>(a.cache.v_slot_data) | reinterpret_cast<uintptr_t>(Wb)) & 15) == 0 &&
                    k_codes_b % 16 == 0 && k_sc_b % 16 == 0 && d.vslot_bytes % 16 == 0 && v_rows == nullptr;
  if (tid == 0) {
    mbar_init(&sm.stg_bar, 1);
    fence_mbar_init();
  }
  int n_batches = 0;    // batches staged so far (mbarrier phase)
  bool stg_failed = false;
  for (int i = 0; i < QN; ++i) {
    const int n_all = sm.nsel[i];
    // more than kRSel selected entries: the apply runs in rounds over the
    // list in the workspace (index order), each round's items in the tables
    const bool multi = n_all > kRSel;
    const int* gl = gsel_base + i * a.sel_stride + 1;
    // end of the round starting at r0: at most kRSel entries, never splitting
    // the K entries of one page (adjacent in an index-ordered list)
    auto round_end = [&](int r0) -> int {
      int r1 = min(n_all, r0 + kRSel);
      if (multi && r1 < n_all) {
        const int en = gl[r1];
        if (en < KG) {
          while (r1 > r0 + 1) {
            const int ep = gl[r1 - 1];
            if (ep < KG && ep / d.SK == en / d.SK) --r1;
            else break;
          }
        }
      }
      return r1;
    };
    // wK of token t of page p: q . R_K summed over the selected slots in mask
    auto wk_of = [&](int p, int mask, int t) -> float {
      const int64_t pg = lhp * d.P + p;
      float acc = 0.f;
      for (int j = 0; j < d.SK; ++j) {
        if (!((mask >> j) & 1)) continue;
        if (a.kw != nullptr) {
          acc += a.kw[((static_cast<int64_t>(bh) * QG + q0 + i) * KG + p * d.SK + j) * kPage + tok_pos(t, a.s_perm)];
          continue;
        }
        const int grp = a.cache.k_slot_group[pg * d.SK + j];
        const uint4 raw = *reinterpret_cast<const uint4*>(a.cache.k_slot_data + (pg * d.SK + j) * d.kslot_bytes + t * 16);
        const float rs = f16_bits_to_f32(a.cache.k_slot_scale[pg * d.SK + j]);
        const uint32_t wds[4] = {raw.x, raw.y, raw.z, raw.w};
        float dot = 0.f;
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          int v = (wds[c >> 3] >> (4 * (c & 7))) & 15;
          v = v > 7 ? v - 16 : v;
          dot = fmaf(sm.Q[i][grp * d.kcg + c], __fmul_rn(static_cast<float>(v), rs), dot);
        }
        acc += dot;
      }
      return acc;
    };
    // selected K slots of page p anywhere in the list (warp-wide; multi-round
    // lists, where a V slot's page may lead a K item of another round)
    auto sel_kmask = [&](int p) -> int {
      int m = 0;
      for (int x = lane; x < n_all; x += 32) {
        const int e = gl[x];
        if (e < KG && e / d.SK == p) m |= 1 << (e - p * d.SK);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m |= __shfl_xor_sync(0xffffffffu, m, o);
      return m;
    };
    // statistics of the exact pass over the selected K pages' valid tokens,
    // per thread: the largest ds, sum of A (e^ds - 1), the token count
    float ex_mx = -INFINITY, ex_zs = 0.f;
    int ex_cov = 0;
    // tables of the round [r0, r1): selected K pages (the first selection of
    // a page leads it) and V slots with the per-item scalars (one round
    // trip), then wK per (selected K page, token), with the exact pass's
    // statistics when `stats` (the logit and q.R_K loads in one round trip)
    auto load_round = [&](int r0, int r1, bool count_reads, bool stats) {
      if (warp == 0) {
        const int nsel = r1 - r0;
        if (multi) {
          if (lane < nsel) sm.sel[i][lane] = gl[r0 + lane];
          __syncwarp();
        }
        const int e = lane < nsel ? sm.sel[i][lane] : -1;
        const bool isk = e >= 0 && e < KG, isv = e >= KG;
        const int p = isk ? e / d.SK : -1;
        const int e_lo = isk ? p * d.SK : 0, e_hi = isk ? e_lo + d.SK : 0;   // the page's K entries
        bool leader = isk;
        int msk = 0;
        for (int k = 0; k < nsel; ++k) {
          const int ek = sm.sel[i][k];
          if (ek >= e_lo && ek < e_hi) {
            if (k < lane) leader = false;
            msk |= 1 << (ek - e_lo);
          }
        }
        const unsigned lt = (1u << lane) - 1u;
        const unsigned bl = __ballot_sync(0xffffffffu, leader);
        const unsigned bv = __ballot_sync(0xffffffffu, isv);
        const unsigned bk = __ballot_sync(0xffffffffu, isk);
        const int nkp_w = __popc(bl);
        if (leader) {
          const int u = __popc(bl & lt);
          const int64_t pg = lhp * d.P + p;
          sm.kp_page[u] = p;
          sm.kp_mask[u] = msk;
          sm.kp_nv[u] = a.cache.valid[pg];
          sm.kp_vm[u] = d.scale_mode == CAREKV_SCALE_INT8 ? f16_bits_to_f32(a.cache.v_master[pg]) : 0.f;
        }
        if (isv) {
          const int v = __popc(bv & lt), ev = e - KG;
          const int pv = ev / d.SV, j = ev % d.SV;
          const int64_t pg = lhp * d.P + pv;
          sm.vsel[v] = ev;
          const int vb = a.cache.v_slot_block[pg * d.SV + j];
          const int t0 = vb * d.vtb;
          sm.vs_t0[v] = t0;
          sm.vs_t1[v] = min(t0 + d.vtb, a.cache.valid[pg]);
          sm.vs_rs[v] = f16_bits_to_f32(a.cache.v_slot_scale[pg * d.SV + j]);
        }
        if (lane == 0) {
          sm.nkp = nkp_w;
          sm.nvs = __popc(bv);
          if (count_reads) {
            reads_k += __popc(bk);
            reads_v += __popc(bv);
          }
        }
      }
      __syncthreads();
      __syncthreads();
      for (int x = tid; x < sm.nkp * kPage; x += NT) {
        const int u = x / kPage, t = x % kPage;
        const int p = sm.kp_page[u], nv = sm.kp_nv[u];
        // the logit is loaded before wK is summed
        const float sv = (stats && !PF && t < nv) ? Sb[i * sst + p * kPage + tok_pos(t, a.s_perm)] : 0.f;
        const float wk = wk_of(p, sm.kp_mask[u], t);
        sm.ds[u][t] = wk;
        if (stats) {
          if (t == 0) ex_cov += nv;
          if (t < nv) {
            const float dsv = __fdiv_rn(wk, a.sqrt_d);
            ex_mx = fmaxf(ex_mx, dsv);
            if (!PF) ex_zs += attw(sv, i) * expm1f(dsv);
          }
        }
      }
      __syncthreads();
    };
    // exact form: shift by the largest ds over the valid tokens of every
    // selected K page (all rounds)
    //
    // The sparse form dO = (cbase O + sum_S cf V) / (cbase + sum_S cf) - O,
    // cf = A cbase (e^ds - 1), takes the tokens outside S through O.  When S
    // holds nearly all the attention and its ds are strongly negative, the
    // new normaliser 1 + sum_S A (e^ds - 1) is tiny and the result rests on
    // O minus the S tokens' share: a few ulps of O's fp32 rounding become
    // errors of 1e-2.  Such a query (normaliser < kIllNorm) takes the direct
    // form instead: the tokens outside S are summed explicitly (A V and A, a
    // pass over their V rows) and S enters with A cbase e^ds, so every term
    // is positive, as in the reference's a_new = A w / sum(A w)
    // (attention.py:96-118).  Decode only (the prefill correction's base
    // output comes from the caller).
    float mshift = 0.f;
    bool ill = false;
    if (exact) {
      int nkp_all = 0;
      ex_mx = -INFINITY;
      ex_zs = 0.f;
      ex_cov = 0;
      for (int q0 = 0; q0 < n_all;) {
        const int q1 = round_end(q0);
        load_round(q0, q1, !multi, true);
        nkp_all += sm.nkp;
        q0 = q1;
        __syncthreads();
      }
      // CTA-wide: max and sum over the warps (the sum only decides the
      // conditioning test), token count
      const float wmx = warp_max(ex_mx), wzs = warp_sum(ex_zs);
      const int wcov = __reduce_add_sync(0xffffffffu, ex_cov);
      if (lane == 0) {
        sm.gv[warp] = wmx;
        sm.gv[NW + warp] = wzs;
        sm.gi[warp] = wcov;
      }
      __syncthreads();
      if (tid == 0) {
        float mx = sm.gv[0], zs = sm.gv[NW];
        int covered = sm.gi[0];
        for (int w = 1; w < NW; ++w) {
          mx = fmaxf(mx, sm.gv[w]);
          zs += sm.gv[NW + w];
          covered += sm.gi[w];
        }
        sm.mshift = (nkp_all == 0) ? 0.f : (covered >= ntot ? mx : fmaxf(mx, 0.f));
        sm.ill = !PF && nkp_all > 0 && covered < ntot && 1.f + zs < kIllNorm;
      }
      __syncthreads();
      mshift = sm.mshift;
      ill = sm.ill != 0;
    }
    const float cbase = exact ? expf(-mshift) : 1.f;
    float num[4] = {0.f, 0.f, 0.f, 0.f};   // channel lane + 32 jj (per-channel decode)
    float acc8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // channels 8 wl + j (word decode)
    float zp = 0.f;
    for (int r0 = 0; r0 < n_all;) {
      const int r1 = round_end(r0);
      if (r0 > 0) __syncthreads();   // every warp is done with the previous round's tables
      if (multi || !exact) load_round(r0, r1, true, false);   // a single round is loaded by the exact pass
      const int nkp = sm.nkp, nvs = sm.nvs, nit = nkp + nvs;
      // batch plan: item -> staging offset, batch boundaries.  A round holds
      // at most kRSel = 32 items: warp 0 scans their sizes, and when they fit
      // one batch the offsets are the exclusive prefix sums; else lane 0
      // packs them greedily in order
      if (warp == 0) {
        const int sz = lane < nit ? (lane < nkp ? k_item_b : v_item_b) : 0;
        int incl = sz;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        if (__shfl_sync(0xffffffffu, incl, 31) <= kRStg) {
          if (lane < nit) sm.ioff[lane] = incl - sz;
          if (lane == 0) {
            sm.bnd[0] = 0;
            sm.bnd[1] = nit;
            sm.nb = 1;
          }
        } else if (lane == 0) {
          int off = 0, nb = 0;
          sm.bnd[0] = 0;
          for (int it = 0; it < nit; ++it) {
            const int isz = it < nkp ? k_item_b : v_item_b;
            if (off + isz > kRStg) {
              sm.bnd[++nb] = it;
              off = 0;
            }
            sm.ioff[it] = off;
            off += isz;
          }
          sm.bnd[++nb] = nit;
          sm.nb = nb;
        }
      }
      __syncthreads();
      const int nb = sm.nb;
      // bulk copies of batch `bt` by the lanes of warp 0 (item per lane)
      auto stage_batch = [&](int bt) {
        if (!bulk || warp != 0) return;
        const int lo = sm.bnd[bt], hi = sm.bnd[bt + 1];
        uint32_t bytes = 0;
        for (int it = lo; it < hi; ++it) bytes += it < nkp ? k_item_b : v_item_b;
        if (lane == 0) mbar_expect_tx(&sm.stg_bar, bytes);
        __syncwarp();
        for (int it = lo + lane; it < hi; it += 32) {
          uint8_t* dst = sm.stg + sm.ioff[it];
          fence_proxy_async();
          if (it < nkp) {
            const int p = sm.kp_page[it];
            const int64_t pg = lhp * d.P + p;
            bulk_g2s(dst, a.cache.v_codes + pg * k_codes_b, k_codes_b, &sm.stg_bar);
            bulk_g2s(dst + k_codes_b, reinterpret_cast<const uint8_t*>(a.cache.v_scale) + pg * k_sc_b, k_sc_b, &sm.stg_bar);
            bulk_g2s(dst + k_codes_b + k_sc_b, Wb + i * sst + p * kPage, kPage * 4, &sm.stg_bar);
          } else {
            const int ev = sm.vsel[it - nkp];
            const int pv = ev / d.SV, j = ev % d.SV;
            const int64_t pg = lhp * d.P + pv;
            bulk_g2s(dst, a.cache.v_slot_data + (pg * d.SV + j) * d.vslot_bytes, d.vslot_bytes, &sm.stg_bar);
            bulk_g2s(dst + d.vslot_bytes, Wb + i * sst + pv * kPage, kPage * 4, &sm.stg_bar);
          }
        }
      };
      stage_batch(0);
    for (int bt = 0; bt < nb; ++bt) {
      if (bt > 0) {
        __syncthreads();   // every warp is done with the previous batch
        stage_batch(bt);
      }
      if (bulk) {
        // bounded wait; the outcome is made CTA-uniform
        stg_failed = __syncthreads_or(!mbar_wait(&sm.stg_bar, n_batches & 1)) != 0;
        if (stg_failed) break;
        ++n_batches;
      }
      for (int item = sm.bnd[bt] + warp; item < sm.bnd[bt + 1]; item += NW) {
        uint8_t* stg = sm.stg + sm.ioff[item];
        if (item < nkp) {
          const int u = item, p = sm.kp_page[u];
          const int64_t pg = lhp * d.P + p;
          const int nv = sm.kp_nv[u];
          const float* vrow = v_rows ? v_rows + (static_cast<int64_t>(h) * a.p_used + p) * kPage * D : nullptr;
          if (!bulk) {
            for (int w = lane; w < (vrow ? 0 : k_codes_b / 4); w += 32)
              reinterpret_cast<uint32_t*>(stg)[w] = reinterpret_cast<const uint32_t*>(a.cache.v_codes + pg * k_codes_b)[w];
            for (int w = lane; w < (vrow ? 0 : k_sc_b); w += 32)
              stg[k_codes_b + w] = reinterpret_cast<const uint8_t*>(a.cache.v_scale)[pg * k_sc_b + w];
            if (lane < kPage)
              reinterpret_cast<float*>(stg + k_codes_b + k_sc_b)[lane] = Wb[i * sst + p * kPage + lane];
            __syncwarp();
          }
          const float* srow = reinterpret_cast<const float*>(stg + k_codes_b + k_sc_b);
          for (int x = lane; x < (vrow ? 0 : kPage * G); x += 32)
            // KIVI scales are exact activation-dtype values (fp32 storage); the
            // uniform base reads its scales back as fp16 (cache.py:713-718)
            sm.stage_sc[warp][x] = d.kivi ? reinterpret_cast<const float*>(stg + k_codes_b)[x]
                                          : read_scale(stg + k_codes_b, x, d.scale_mode, sm.kp_vm[u]);
          float cf = 0.f;
          if (lane < kPage && lane < nv) {
            const float A = attw(srow[tok_pos(lane, a.s_perm)], i);
            const float wk = sm.ds[u][lane];
            if (exact) {
              const float dsv = __fdiv_rn(wk, a.sqrt_d);
              // direct form (ill): the S token's own new weight A e^(ds - m)
              cf = ill ? A * (dsv <= 80.f ? cbase * expf(dsv) : expf(dsv - mshift))
                       : A * (dsv <= 80.f ? cbase * expm1f(dsv) : expf(dsv - mshift) - cbase);
            } else {
              cf = A * wk * rp.k_corr_scale;
            }
          }
          if (lane < kPage) sm.coef[warp][lane] = cf;
          zp += warp_sum(cf);
          __syncwarp();
          if (vrow) {   // base V rows given by the caller
            for (int t = 0; t < nv; ++t) {
              const float c = sm.coef[warp][t];
#pragma unroll
              for (int jj = 0; jj < 4; ++jj) {
                const int ch = lane + 32 * jj;
                if (ch < D) num[jj] = fmaf(c, vrow[t * D + ch], num[jj]);
              }
            }
          } else if (fast3) {
            for (int t = rg; t < nv; t += RG) {
              const float sg = sm.stage_sc[warp][t * G + (8 * wl) / d.gsize];
              acc_int3_word(stg + t * R, wl, pack_h2(sg, sg), sm.coef[warp][t], acc8);
            }
          } else {
            for (int t = 0; t < nv; ++t) {
              const float c = sm.coef[warp][t];
#pragma unroll
              for (int jj = 0; jj < 4; ++jj) {
                const int ch = lane + 32 * jj;
                if (ch < D) {
                  const int cv = unpack_code(stg + t * R, ch, d.bits);
                  const float sc = sm.stage_sc[warp][t * G + ch / d.gsize];
                  // KIVI: V_hat rounded in the activation dtype, then fp16
                  const float vh = d.kivi ? f16r(kivi_hat(cv, sc, a.dt)) : f16r(__fmul_rn(static_cast<float>(cv), sc));
                  num[jj] = fmaf(c, vh, num[jj]);
                }
              }
            }
          }
        } else {
          const int v = item - nkp;
          const int ev = sm.vsel[v];
          const int p = ev / d.SV, j = ev % d.SV;
          const int t0 = sm.vs_t0[v], t1 = sm.vs_t1[v];
          if (!bulk) {
            const int64_t pg = lhp * d.P + p;
            const uint32_t* src = reinterpret_cast<const uint32_t*>(a.cache.v_slot_data + (pg * d.SV + j) * d.vslot_bytes);
            for (int w = lane; w < d.vslot_bytes / 4; w += 32) reinterpret_cast<uint32_t*>(stg)[w] = src[w];
            if (lane < kPage)
              reinterpret_cast<float*>(stg + d.vslot_bytes)[lane] = Wb[i * sst + p * kPage + lane];
            __syncwarp();
          }
          const float* srow = reinterpret_cast<const float*>(stg + d.vslot_bytes);
          const float rs = sm.vs_rs[v];
          int u = -1;
          for (int x = 0; x < nkp; ++x) if (sm.kp_page[x] == p) u = x;
          // the page's selected K slots led by an item of another round
          const int omask = (exact && multi && u < 0) ? sel_kmask(p) : 0;
          if (lane < d.vtb) {
            const int t = t0 + lane;
            float cf = 0.f;
            if (t < t1) {
              const float A = attw(srow[tok_pos(t, a.s_perm)], i);
              float w = 1.f;
              if (exact) {
                const float dsv = u >= 0 ? __fdiv_rn(sm.ds[u][t], a.sqrt_d)
                                         : (omask ? __fdiv_rn(wk_of(p, omask, t), a.sqrt_d) : 0.f);
                w = dsv <= 80.f ? cbase * expf(dsv) : expf(dsv - mshift);
              }
              cf = A * w;
            }
            sm.coef[warp][lane] = cf;
          }
          __syncwarp();
          // row r of the payload: D/2 bytes, channel c at nibble c of the row
          const uint32_t* pay = reinterpret_cast<const uint32_t*>(stg);
          for (int r = rg; r < t1 - t0; r += RG) acc_nib_word(pay[r * WPR + wl], sm.coef[warp][r] * rs, acc8);
        }
        __syncwarp();
      }
    }
      if (stg_failed) break;
      r0 = r1;
    }
    if (stg_failed) {
      // the staging copies did not land in time: flag it, let the copies in
      // flight land (bounded) before the CTA exits, keep the base output
      if (tid == 0) {
        atomicOr(a.cache.error_flag, 4);
        (void)mbar_wait(&sm.stg_bar, n_batches & 1);
      }
      __syncthreads();
      write_base();
      return;
    }
    if (ill) {
      // direct form: A V and A of every valid token outside the selected K
      // pages (a page bitmap at the end of the staging area, free after the
      // rounds)
      const int nwords = (a.p_used + 31) >> 5;
      uint32_t* kbits = reinterpret_cast<uint32_t*>(sm.stg + kRStg) - nwords;
      __syncthreads();
      for (int x = tid; x < nwords; x += NT) kbits[x] = 0u;
      __syncthreads();
      for (int x = tid; x < n_all; x += NT) {
        const int e = multi ? gl[x] : sm.sel[i][x];
        if (e < KG) atomicOr(&kbits[(e / d.SK) >> 5], 1u << ((e / d.SK) & 31));
      }
      __syncthreads();
      // Lane l decodes channels 4l .. 4l+3 of every row (one scale group).
      // Warp w takes the pages p = w (mod NW) in ascending order, so per
      // channel the pages and rows are summed in the same order whichever way
      // the rows arrive.
      float o2[4] = {0.f, 0.f, 0.f, 0.f}, z2 = 0.f;
      DirectLane dl;
      dl.rs = D == 64 ? 2 : 1;                  // D = 64: half-warps on alternate rows
      dl.half = dl.rs == 2 ? lane >> 4 : 0;
      dl.cb = 4 * (dl.rs == 2 ? (lane & 15) : lane);   // first channel of the lane
      dl.cl = dl.cb < D;
      dl.b0 = dl.cb * d.bits;                   // its bit offset in a packed row
      dl.wsh = dl.b0 & 31;
      dl.two = dl.wsh + 4 * d.bits > 32;        // the 4 codes straddle a 32-bit word
      dl.cmask = (1u << d.bits) - 1u;
      dl.csign = 1u << (d.bits - 1);
      const int cb = dl.cb;
      const bool cl = dl.cl;
      // staged: batches of pages copied into shared memory by warp 0's
      // lanes (packed V rows, V scales, logits; one round trip per batch),
      // a multiple of NW pages per batch to keep each warp's page order
      const int pbytes = k_codes_b + k_sc_b + kPage * 4;
      const int cap = min(32, (kRStg - nwords * 4) / pbytes) / NW * NW;
      const bool staged = bulk && cap > 0;
      const int step = staged ? cap : NW;   // unstaged: warp w reads page p0 + w from global memory
      for (int p0 = 0; p0 < np; p0 += step) {
        const int p1 = min(np, p0 + step);
        if (staged) {
          __syncthreads();   // every warp is done with the previous batch
          if (warp == 0) {
            const int p = p0 + lane;
            const bool take = p < p1 && !((kbits[p >> 5] >> (p & 31)) & 1u);
            const unsigned tm = __ballot_sync(0xffffffffu, take);
            const int64_t pg = lhp * d.P + p;
            if (lane == 0) mbar_expect_tx(&sm.stg_bar, static_cast<uint32_t>(__popc(tm) * pbytes));
            __syncwarp();
            if (take) {
              uint8_t* dst = sm.stg + lane * pbytes;
              fence_proxy_async();
              bulk_g2s(dst, a.cache.v_codes + pg * k_codes_b, k_codes_b, &sm.stg_bar);
              bulk_g2s(dst + k_codes_b, reinterpret_cast<const uint8_t*>(a.cache.v_scale) + pg * k_sc_b, k_sc_b, &sm.stg_bar);
              bulk_g2s(dst + k_codes_b + k_sc_b, Wb + i * sst + p * kPage, kPage * 4, &sm.stg_bar);
            }
            // the pages' row counts and masters while the copies are in flight
            if (lane < cap) {
              sm.kp_nv[lane] = take ? a.cache.valid[pg] : 0;
              sm.kp_vm[lane] = take && d.scale_mode == CAREKV_SCALE_INT8 ? f16_bits_to_f32(a.cache.v_master[pg]) : 0.f;
            }
          }
          stg_failed = __syncthreads_or(!mbar_wait(&sm.stg_bar, n_batches & 1)) != 0;
          if (stg_failed) break;
          ++n_batches;
        }
        for (int x = warp; x < p1 - p0; x += NW) {
          const int p = p0 + x;
          const uint8_t* rows;
          const uint8_t* scl;
          int nv;
          float vm, sv;
          if (staged) {
            nv = sm.kp_nv[x];   // 0 for the selected pages
            if (nv == 0) continue;
            rows = sm.stg + x * pbytes;
            scl = rows + k_codes_b;
            vm = sm.kp_vm[x];
            sv = reinterpret_cast<const float*>(rows + k_codes_b + k_sc_b)[tok_pos(lane & 15, a.s_perm)];
          } else {
            if ((kbits[p >> 5] >> (p & 31)) & 1u) continue;
            const int64_t pg = lhp * d.P + p;
            nv = a.cache.valid[pg];
            vm = d.scale_mode == CAREKV_SCALE_INT8 ? f16_bits_to_f32(a.cache.v_master[pg]) : 0.f;
            rows = a.cache.v_codes + pg * k_codes_b;
            scl = reinterpret_cast<const uint8_t*>(a.cache.v_scale) + pg * k_sc_b;
            // every logit row exists up to p_used
            sv = Sb[i * sst + p * kPage + tok_pos(lane & 15, a.s_perm)];
          }
          const float At = (lane & 15) < nv ? attw(sv, i) : 0.f;
          direct_rows(d, a.dt, dl, rows, scl, vm, nv, At, o2, z2);
        }
      }
      if (dl.rs == 2) {   // the odd rows' sums (lanes 16..31) onto lanes 0..15
#pragma unroll
        for (int k = 0; k < 4; ++k) o2[k] += __shfl_down_sync(0xffffffffu, o2[k], 16);
        z2 += __shfl_down_sync(0xffffffffu, z2, 16);
      }
      if (cl && dl.half == 0) {
#pragma unroll
        for (int k = 0; k < 4; ++k) sm.acc2[warp][cb + k] = o2[k];
      }
      if (lane == 0) sm.z2[warp] = z2;
      if (stg_failed) {
        // a staged batch did not land in time: as for the rounds above
        if (tid == 0) {
          atomicOr(a.cache.error_flag, 4);
          (void)mbar_wait(&sm.stg_bar, n_batches & 1);
        }
        __syncthreads();
        write_base();
        return;
      }
    }
    // fold the word layout's row groups onto lanes 0 .. WPR-1
    for (int o = WPR; o < 32; o <<= 1)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc8[j] += __shfl_xor_sync(0xffffffffu, acc8[j], o);
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int c = lane + 32 * jj;
      if (c < D) sm.acc[warp][c] = num[jj];
    }
    __syncwarp();
    if (lane < WPR)
#pragma unroll
      for (int j = 0; j < 8; ++j) sm.acc[warp][8 * lane + j] += acc8[j];
    if (lane == 0) sm.z[warp] = zp;
    __syncthreads();
    if (tid < D) {
      float n = 0.f, z = 0.f;
      for (int w = 0; w < NW; ++w) { n += sm.acc[w][tid]; z += sm.z[w]; }
      const float ob = sm.O[i][tid];
      // exact form: a_new @ V = (cbase * sum_t A V + num) / (cbase * sum_t A + z); sum_t A V and
      // sum_t A are O and 1 in decode, given by the caller in the prefill correction
      const int64_t row = static_cast<int64_t>(bh) * QG + q0 + i;
      const float oe = o_exact ? o_exact[row * D + tid] : ob;
      const float as = (po_direct && a.pl) ? a.pl[row] : 1.f;
      float delta;
      if (ill) {
        // direct form: (cbase sum_notS A V + sum_S A cbase e^ds V) / (cbase sum_notS A + sum_S A cbase e^ds)
        float on = 0.f, zn = 0.f;
        for (int w = 0; w < NW; ++w) { on += sm.acc2[w][tid]; zn += sm.z2[w]; }
        delta = __fdiv_rn(fmaf(cbase, on, n), fmaf(cbase, zn, z)) - ob;
      } else {
        delta = exact ? (__fdiv_rn(fmaf(cbase, oe, n), fmaf(cbase, as, z)) - ob) : (n - z * ob);
      }
      store_act(a.out, (static_cast<int64_t>(s) * Hq + h * QG + q0 + i) * D + tid, ob + delta, a.dt);
    }
    __syncthreads();
  }
  if (a.cache.read_counter != nullptr && tid == 0) {
    unsigned long long* rc = a.cache.read_counter + (static_cast<int64_t>(a.layer) * d.H + h) * 2;
    if (sm.any_k && reads_k) atomicAdd(rc, static_cast<unsigned long long>(reads_k));
    if (reads_v) atomicAdd(rc + 1, static_cast<unsigned long long>(reads_v));
  }
}

}  // namespace carekv
