// Decode attention over the packed cache (kernels K3, K4 and K2).
//
// decode_partial_kernel  (K3)  split-K pass: each CTA streams a range of
//   pages of one (sequence, kv head), dequantizes K and V rows to their fp16
//   values, computes the logits of the kv head's query group, keeps an online
//   softmax and the weighted V sum, writes the logits to the workspace (the
//   router needs the normalised weights of every token) and one (m, l, O)
//   partial per CTA.
// route_kernel  (K4 + K2)  per (sequence, kv head): merges the partials into
//   O_base, scores every stored residual slot (combined_kvscore or the sketch
//   proxy), normalises per query, selects the joint / separate top-k and
//   applies the exact softmax renormalisation (or the linear form), writing
//   O = O_base + dO.
//
// Reference: attention.py:979-1039 (base decode), attention.py:576-957
// (vectorized_joint_correction), attention.py:96-118 and 167-184,
// residual_router.py:37-76.
#include "common.cuh"
#include "internal.h"

namespace carekv {

struct DecodeArgs {
  carekv_config_t cfg;
  carekv_cache_t cache;
  int layer;
  const void* q;
  void* out;
  int dt;
  int seq_begin;
  int qn;           // query heads per kv head
  int pps;          // pages per split
  int n_splits;
  int p_used;       // workspace page stride
  float sf;         // fp32(1/sqrt(D))
  float sqrt_d;     // fp32(sqrt(D))
  float* S;         // [bh][qn][p_used*16] logits
  float* pm;        // [bh][n_splits][qn]
  float* pl;
  float* po;        // [bh][n_splits][qn][D]
  float* scores;    // [bh][qn][p_used*(SK+SV)]
  int* sel_out;     // [bh][qn][1 + kMaxSel]: count, then selected grid indices
  const float* sketch_proj;
  carekv_route_params_t rp;
};

// ─────────────────────────── K3: split-K pass ───────────────────────────
template <int QN, int DPL>
__global__ void __launch_bounds__(128) decode_partial_kernel(DecodeArgs a) {
  const Dims d = make_dims(a.cfg);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int bh = blockIdx.x, split = blockIdx.y;
  const int s = bh / d.H, h = bh % d.H, b = a.seq_begin + s;
  const int D = d.D;
  const int64_t lhp = d.lhp(b, a.layer, h);
  const int np = min(a.cache.num_pages[lhp], a.p_used);
  const int p0 = split * a.pps, p1 = min(np, p0 + a.pps);
  const int Hq = d.H * QN;

  float q[QN][DPL];
#pragma unroll
  for (int i = 0; i < QN; ++i)
#pragma unroll
    for (int j = 0; j < DPL; ++j)
      q[i][j] = load_act(a.q, (static_cast<int64_t>(s) * Hq + h * QN + i) * D + lane + 32 * j, a.dt);

  float m[QN], l[QN], o[QN][DPL];
#pragma unroll
  for (int i = 0; i < QN; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int j = 0; j < DPL; ++j) o[i][j] = 0.f;
  }
  float* Srow = a.S + static_cast<int64_t>(bh) * QN * a.p_used * kPage;
  const int64_t sstride = static_cast<int64_t>(a.p_used) * kPage;

  for (int p = p0 + warp; p < p1; p += 4) {
    const int64_t pg = lhp * d.P + p;
    const int nv = a.cache.valid[pg];
    float mk = 0.f, mv = 0.f;
    if (d.scale_mode == CAREKV_SCALE_INT8) {
      mk = f16_bits_to_f32(a.cache.k_master[pg]);
      mv = f16_bits_to_f32(a.cache.v_master[pg]);
    }
    for (int t = 0; t < nv; ++t) {
      const uint8_t* kr = a.cache.k_codes + (pg * kPage + t) * d.R;
      const uint8_t* vr = a.cache.v_codes + (pg * kPage + t) * d.R;
      const int64_t srow = (pg * kPage + t) * d.G;
      float kh[DPL], vh[DPL];
#pragma unroll
      for (int j = 0; j < DPL; ++j) {
        const int c = lane + 32 * j;
        const int g = c / d.gsize;
        const float sk = read_scale(a.cache.k_scale, srow + g, d.scale_mode, mk);
        const float sv = read_scale(a.cache.v_scale, srow + g, d.scale_mode, mv);
        kh[j] = f16r(__fmul_rn(static_cast<float>(unpack_code(kr, c, d.bits)), sk));
        vh[j] = f16r(__fmul_rn(static_cast<float>(unpack_code(vr, c, d.bits)), sv));
      }
#pragma unroll
      for (int i = 0; i < QN; ++i) {
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < DPL; ++j) acc = fmaf(kh[j], q[i][j], acc);
        const float sc = __fmul_rn(warp_sum(acc), a.sf);
        if (lane == 0) Srow[i * sstride + p * kPage + t] = sc;
        const float mn = fmaxf(m[i], sc);
        const float corr = expf(m[i] - mn);  // m = -inf on the first token -> 0
        const float e = expf(sc - mn);
        l[i] = l[i] * corr + e;
#pragma unroll
        for (int j = 0; j < DPL; ++j) o[i][j] = fmaf(o[i][j], corr, e * vh[j]);
        m[i] = mn;
      }
    }
  }

  // merge the 4 warps
  __shared__ float sm_m[4][QN], sm_l[4][QN];
  __shared__ float sm_o[4][QN][DPL * 32];
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < QN; ++i) { sm_m[warp][i] = m[i]; sm_l[warp][i] = l[i]; }
  }
#pragma unroll
  for (int i = 0; i < QN; ++i)
#pragma unroll
    for (int j = 0; j < DPL; ++j) sm_o[warp][i][lane + 32 * j] = o[i][j];
  __syncthreads();
  const int64_t part = static_cast<int64_t>(bh) * a.n_splits + split;
  for (int idx = threadIdx.x; idx < QN * D; idx += blockDim.x) {
    const int i = idx / D, c = idx % D;
    float M = -INFINITY;
    for (int w = 0; w < 4; ++w) M = fmaxf(M, sm_m[w][i]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
      for (int w = 0; w < 4; ++w) {
        const float f = sm_m[w][i] == -INFINITY ? 0.f : expf(sm_m[w][i] - M);
        L += sm_l[w][i] * f;
        O += sm_o[w][i][c] * f;
      }
    }
    a.po[(part * QN + i) * D + c] = O;
    if (c == 0) {
      a.pm[part * QN + i] = M;
      a.pl[part * QN + i] = L;
    }
  }
}

// ─────────────────────────── K4 + K2: route ───────────────────────────
constexpr int kMaxSel = 32;  // selected slots per query (host-validated)
constexpr float kEps = 1e-6f;

__device__ __forceinline__ bool better(float s1, int i1, float s2, int i2) {
  return s1 > s2 || (s1 == s2 && i1 < i2);
}

template <int QN>
__global__ void __launch_bounds__(256) route_kernel(DecodeArgs a) {
  const Dims d = make_dims(a.cfg);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nwarp = blockDim.x >> 5;
  const int bh = blockIdx.x;
  const int s = bh / d.H, h = bh % d.H, b = a.seq_begin + s;
  const int D = d.D;
  const int Hq = d.H * QN;
  const int64_t lhp = d.lhp(b, a.layer, h);
  const int np = min(a.cache.num_pages[lhp], a.p_used);
  const carekv_route_params_t& rp = a.rp;

  __shared__ float sQ[QN][128], sO[QN][128], sM[QN], sL[QN];
  __shared__ float red[32][QN], red2[32][QN], nk_s[QN], nv_s[QN];
  __shared__ int sel[QN][kMaxSel];
  __shared__ float selv[QN][kMaxSel];
  __shared__ float ds_sm[QN][kMaxSel][kPage];
  __shared__ int kp_sm[QN][kMaxSel];
  __shared__ int nsel[QN];
  __shared__ int cnt_k, cnt_v, any_k;
  __shared__ float redf[32];
  __shared__ int redi[32];

  for (int idx = tid; idx < QN * D; idx += blockDim.x) {
    const int i = idx / D, c = idx % D;
    sQ[i][c] = load_act(a.q, (static_cast<int64_t>(s) * Hq + h * QN + i) * D + c, a.dt);
  }
  // combine split partials
  if (tid < QN) {
    float M = -INFINITY;
    for (int sp = 0; sp < a.n_splits; ++sp) M = fmaxf(M, a.pm[(static_cast<int64_t>(bh) * a.n_splits + sp) * QN + tid]);
    float L = 0.f;
    if (M != -INFINITY)
      for (int sp = 0; sp < a.n_splits; ++sp) {
        const int64_t k = (static_cast<int64_t>(bh) * a.n_splits + sp) * QN + tid;
        if (a.pm[k] != -INFINITY) L += a.pl[k] * expf(a.pm[k] - M);
      }
    sM[tid] = M;
    sL[tid] = L;
  }
  __syncthreads();
  for (int idx = tid; idx < QN * D; idx += blockDim.x) {
    const int i = idx / D, c = idx % D;
    float O = 0.f;
    if (sL[i] > 0.f) {
      for (int sp = 0; sp < a.n_splits; ++sp) {
        const int64_t k = (static_cast<int64_t>(bh) * a.n_splits + sp) * QN + i;
        if (a.pm[k] != -INFINITY) O += a.po[k * D + c] * expf(a.pm[k] - sM[i]);
      }
      O = __fdiv_rn(O, sL[i]);
    }
    sO[i][c] = O;
  }
  if (tid == 0) { cnt_k = 0; cnt_v = 0; any_k = 0; }
  __syncthreads();

  auto write_base = [&]() {
    if (tid < QN) a.sel_out[(static_cast<int64_t>(bh) * QN + tid) * (kMaxSel + 1)] = 0;
    for (int idx = tid; idx < QN * D; idx += blockDim.x) {
      const int i = idx / D, c = idx % D;
      store_act(a.out, (static_cast<int64_t>(s) * Hq + h * QN + i) * D + c, sO[i][c], a.dt);
    }
  };
  if (np == 0 || rp.kind == CAREKV_KIND_NONE) { write_base(); return; }

  const int KG = a.p_used * d.SK;        // K grid entries
  const int VG = a.p_used * d.SV;
  const int NG = KG + VG;
  float* sc = a.scores + static_cast<int64_t>(bh) * QN * NG;
  const float* Sb = a.S + static_cast<int64_t>(bh) * QN * a.p_used * kPage;
  const int64_t sstride = static_cast<int64_t>(a.p_used) * kPage;

  // ── count stored slots (the reference's index builders) ──
  int ck = 0, cv = 0;
  for (int e = tid; e < np * d.SK; e += blockDim.x) {
    const int64_t pg = lhp * d.P + e / d.SK;
    ck += (a.cache.k_slot_group[pg * d.SK + e % d.SK] >= 0) && a.cache.valid[pg] > 0;
  }
  for (int e = tid; e < np * d.SV; e += blockDim.x) {
    const int64_t pg = lhp * d.P + e / d.SV;
    const int vb = a.cache.v_slot_block[pg * d.SV + e % d.SV];
    cv += (vb >= 0) && (min(vb * d.vtb + d.vtb, a.cache.valid[pg]) > vb * d.vtb);
  }
  atomicAdd(&cnt_k, ck);
  atomicAdd(&cnt_v, cv);
  __syncthreads();
  const int n_k = cnt_k, n_v = cnt_v;
  const bool want_k = (rp.kind == CAREKV_KIND_BOTH || rp.kind == CAREKV_KIND_K) && n_k > 0;
  const bool want_v = (rp.kind == CAREKV_KIND_BOTH || rp.kind == CAREKV_KIND_V) && n_v > 0;
  int bk = 0, bv = 0;
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
  if ((!want_k && !want_v) || (bk == 0 && bv == 0)) { write_base(); return; }
  const bool score_k = want_k && bk > 0;
  const bool score_v = want_v && bv > 0;

  // ── K scores: one warp per grid entry (attention.py:704-725) ──
  for (int e = warp; e < KG; e += nwarp) {
    const int p = e / d.SK, j = e % d.SK;
    float* dst = sc + e;
    const int64_t pg = lhp * d.P + p;
    const int grp = p < np ? a.cache.k_slot_group[pg * d.SK + j] : -1;
    const int nv = p < np ? a.cache.valid[pg] : 0;
    if (!score_k || grp < 0 || nv == 0) {
      if (lane < QN) dst[lane * NG] = -1.f;
      continue;
    }
    const uint8_t* pay = a.cache.k_slot_data + (pg * d.SK + j) * d.kslot_bytes;
    const float rs = f16_bits_to_f32(a.cache.k_slot_scale[pg * d.SK + j]);
    const int t = lane >> 1, half = lane & 1;   // 16 tokens x 2 channel halves
    float r[16];
#pragma unroll
    for (int c = 0; c < 16; ++c) r[c] = unpack_nibble(pay, t * 32 + half * 16 + c, rs);
    const int c0 = grp * d.kcg + half * 16;
    if (rp.kscore_live) {
      const float vc = sqrtf(a.cache.v_norm2[pg]);
#pragma unroll
      for (int i = 0; i < QN; ++i) {
        float dot = 0.f;
#pragma unroll
        for (int c = 0; c < 16; ++c) dot = fmaf(sQ[i][c0 + c], r[c], dot);
        dot += __shfl_xor_sync(0xffffffffu, dot, 1);
        float term = 0.f;
        if (t < nv) {
          const float dS = __fdiv_rn(dot, a.sqrt_d);
          const float A = __fdiv_rn(expf(Sb[i * sstride + p * kPage + t] - sM[i]), sL[i]);
          term = dS * (A * (1.f - A));
        }
        float ss = half == 0 ? term * term : 0.f;
        ss = warp_sum(ss);
        float ks = sqrtf(ss) * vc;
        if (!(ks == ks) || isinf(ks)) ks = 0.f;
        ks = fmaxf(ks, 0.f);
        if (lane == 0) dst[i * NG] = ks * rp.sensitivity;
      }
    } else {
      // proxy: mass * |q_sketch . k_sketch| * boundary * vdiff * sens
      for (int i = 0; i < QN; ++i) {
        float A = 0.f, inv = 0.f, vd = 0.f;
        if (t < nv && half == 0) {
          const float st = Sb[i * sstride + p * kPage + t];
          A = __fdiv_rn(expf(st - sM[i]), sL[i]);
          inv = __fdiv_rn(1.f, fmaxf(sM[i] - st, kEps));
          // ||V_hat_t - O_base||
          const uint8_t* vr = a.cache.v_codes + (pg * kPage + t) * d.R;
          const float mv = d.scale_mode == CAREKV_SCALE_INT8 ? f16_bits_to_f32(a.cache.v_master[pg]) : 0.f;
          float acc = 0.f;
          for (int c = 0; c < D; ++c) {
            const float svv = read_scale(a.cache.v_scale, (pg * kPage + t) * d.G + c / d.gsize, d.scale_mode, mv);
            const float df = f16r(__fmul_rn(static_cast<float>(unpack_code(vr, c, d.bits)), svv)) - sO[i][c];
            acc = fmaf(df, df, acc);
          }
          vd = sqrtf(acc);
        }
        const float mass = warp_sum(A);
        const float bnd = warp_sum(A * inv);
        const float pvd = warp_sum(A * vd);
        float qd = 0.f;
        if (lane < d.sketch && a.cache.k_sketch != nullptr) {
          float qs = 0.f;
          for (int c = 0; c < d.kcg; ++c) qs = fmaf(sQ[i][grp * d.kcg + c], a.sketch_proj[c * d.sketch + lane], qs);
          qd = qs * f16_bits_to_f32(a.cache.k_sketch[(pg * d.C + grp) * d.sketch + lane]);
        }
        qd = fabsf(warp_sum(qd));
        if (lane == 0) dst[i * NG] = mass * qd * bnd * pvd * rp.sensitivity;
      }
    }
  }
  // ── V scores: one thread per grid entry (attention.py:787-790) ──
  for (int e = tid; e < VG; e += blockDim.x) {
    const int p = e / d.SV, j = e % d.SV;
    const int64_t pg = lhp * d.P + p;
    const int vb = p < np ? a.cache.v_slot_block[pg * d.SV + j] : -1;
    const int nv = p < np ? a.cache.valid[pg] : 0;
    const int t0 = vb * d.vtb, t1 = min(t0 + d.vtb, nv);
    for (int i = 0; i < QN; ++i) {
      float v = -1.f;
      if (score_v && vb >= 0 && t1 > t0) {
        float mass = 0.f;
        for (int t = t0; t < t1; ++t) mass += __fdiv_rn(expf(Sb[i * sstride + p * kPage + t] - sM[i]), sL[i]);
        v = __fmul_rn(__fmul_rn(mass, f16_bits_to_f32(a.cache.v_err[pg * d.NV + vb])), rp.sensitivity);
      }
      sc[i * NG + KG + e] = v;
    }
  }
  __syncthreads();

  // ── per-query normalisation (attention.py:830-844) ──
  if (rp.score_normalize && rp.kind == CAREKV_KIND_BOTH && score_k && score_v) {
    for (int i = 0; i < QN; ++i) {
      float ak = 0.f, av = 0.f;
      for (int e = tid; e < NG; e += blockDim.x) {
        const float v = sc[i * NG + e];
        if (v >= 0.f) { if (e < KG) ak += v; else av += v; }
      }
      ak = warp_sum(ak);
      av = warp_sum(av);
      if (lane == 0) { red[warp][i] = ak; red2[warp][i] = av; }
    }
    __syncthreads();
    if (tid < QN) {
      float x = 0.f, y = 0.f;
      for (int w = 0; w < nwarp; ++w) { x += red[w][tid]; y += red2[w][tid]; }
      nk_s[tid] = fmaxf(__fdiv_rn(x, static_cast<float>(n_k)), kEps);
      nv_s[tid] = fmaxf(__fdiv_rn(y, static_cast<float>(n_v)), kEps);
    }
    __syncthreads();
    for (int e = tid; e < NG; e += blockDim.x)
      for (int i = 0; i < QN; ++i) {
        const float v = sc[i * NG + e];
        if (v >= 0.f) {
          float r = e < KG ? __fdiv_rn(v, nk_s[i]) : __fdiv_rn(v, nv_s[i]);
          if (rp.kscore_live) r = __fmul_rn(r, e < KG ? rp.lambda_k : rp.lambda_v);
          sc[i * NG + e] = r;
        }
      }
    __syncthreads();
  }

  // ── top-k selection, ties -> lower grid index (attention.py:856-875) ──
  const bool joint = rp.joint && rp.kind == CAREKV_KIND_BOTH && score_k && score_v;
  auto pick = [&](int i, int lo, int hi, int k) {
    for (int r = 0; r < k; ++r) {
      float best = -1.f;
      int bi = 0x7fffffff;
      for (int e = lo + tid; e < hi; e += blockDim.x) {
        const float v = sc[i * NG + e];
        if (v >= 0.f && better(v, e, best, bi)) { best = v; bi = e; }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(ob, oi, best, bi)) { best = ob; bi = oi; }
      }
      if (lane == 0) { redf[warp] = best; redi[warp] = bi; }
      __syncthreads();
      if (tid == 0) {
        float bb = -1.f;
        int ii = 0x7fffffff;
        for (int w = 0; w < nwarp; ++w)
          if (better(redf[w], redi[w], bb, ii)) { bb = redf[w]; ii = redi[w]; }
        if (bb >= 0.f && nsel[i] < kMaxSel) {
          selv[i][nsel[i]] = bb;
          sel[i][nsel[i]++] = ii;
          sc[i * NG + ii] = -2.f;
          if (ii < KG) any_k = 1;
        }
      }
      __syncthreads();
    }
  };
  if (tid < QN) nsel[tid] = 0;
  __syncthreads();
  for (int i = 0; i < QN; ++i) {
    if (joint) {
      const int mb = (bk > 0 && bv > 0) ? bk + bv : max(bk, bv);
      pick(i, 0, NG, min(mb, n_k + n_v));
    } else {
      if (score_k) pick(i, 0, KG, bk);
      if (score_v) pick(i, KG, NG, bv);
    }
  }
  __syncthreads();
  // restore the picked scores and publish the selection (parity readback)
  if (tid < QN) {
    int* so = a.sel_out + (static_cast<int64_t>(bh) * QN + tid) * (kMaxSel + 1);
    so[0] = nsel[tid];
    for (int k = 0; k < nsel[tid]; ++k) {
      so[1 + k] = sel[tid][k];
      sc[tid * NG + sel[tid][k]] = selv[tid][k];
    }
  }

  // ── apply (attention.py:877-943, 96-118): one warp per query ──
  const bool exact = rp.exact && any_k;
  int reads_k = 0, reads_v = 0;
  for (int i = warp; i < QN; i += nwarp) {
    float num[4] = {0.f, 0.f, 0.f, 0.f};  // per lane channels lane + 32*jj
    // distinct K pages of this query with their summed q.R_K per token
    int nkp = 0;
    for (int k = 0; k < nsel[i]; ++k) {
      const int e = sel[i][k];
      if (e >= KG) continue;
      ++reads_k;
      const int p = e / d.SK;
      int slot = -1;
      for (int u = 0; u < nkp; ++u) if (kp_sm[i][u] == p) slot = u;
      if (slot < 0) {
        slot = nkp++;
        if (lane == 0) kp_sm[i][slot] = p;
        if (lane < kPage) ds_sm[i][slot][lane] = 0.f;
      }
      __syncwarp();
      const int64_t pg = lhp * d.P + p;
      const int j = e % d.SK;
      const int grp = a.cache.k_slot_group[pg * d.SK + j];
      const uint8_t* pay = a.cache.k_slot_data + (pg * d.SK + j) * d.kslot_bytes;
      const float rs = f16_bits_to_f32(a.cache.k_slot_scale[pg * d.SK + j]);
      if (lane < kPage) {
        float dot = 0.f;
        for (int c = 0; c < d.kcg; ++c) dot = fmaf(sQ[i][grp * d.kcg + c], unpack_nibble(pay, lane * d.kcg + c, rs), dot);
        ds_sm[i][slot][lane] += dot;  // wK (unscaled), summed over this page's selected groups
      }
      __syncwarp();
    }
    // exact: shift by m = max ds (>= 0 unless every token carries a K slot)
    float mshift = 0.f;
    float z = 1.f;
    if (exact) {
      float mx = -INFINITY;
      int covered = 0;
      for (int u = 0; u < nkp; ++u) {
        const int64_t pg = lhp * d.P + kp_sm[i][u];
        const int nv = a.cache.valid[pg];
        covered += nv;
        for (int t = 0; t < nv; ++t) mx = fmaxf(mx, __fdiv_rn(ds_sm[i][u][t], a.sqrt_d));
      }
      int ntot = 0;
      for (int p = lane; p < np; p += 32) ntot += a.cache.valid[lhp * d.P + p];
      for (int o = 16; o > 0; o >>= 1) ntot += __shfl_xor_sync(0xffffffffu, ntot, o);
      mshift = (nkp == 0) ? 0.f : (covered >= ntot ? mx : fmaxf(mx, 0.f));
      const float cbase = expf(-mshift);
      z = cbase;
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int c = lane + 32 * jj;
        if (c < D) num[jj] = cbase * sO[i][c];
      }
    }
    const float cbase = expf(-mshift);
    // K pages: A_t * d_t * V_hat_t (exact) or A_t * wK_t * (V_hat_t - O) (linear)
    for (int u = 0; u < nkp; ++u) {
      const int p = kp_sm[i][u];
      const int64_t pg = lhp * d.P + p;
      const int nv = a.cache.valid[pg];
      const float mv = d.scale_mode == CAREKV_SCALE_INT8 ? f16_bits_to_f32(a.cache.v_master[pg]) : 0.f;
      for (int t = 0; t < nv; ++t) {
        const float A = __fdiv_rn(expf(Sb[i * sstride + p * kPage + t] - sM[i]), sL[i]);
        const float wk = ds_sm[i][u][t];
        float coef;
        if (exact) {
          const float dsv = __fdiv_rn(wk, a.sqrt_d);
          const float dt_ = dsv <= 80.f ? cbase * expm1f(dsv) : expf(dsv - mshift) - cbase;
          coef = A * dt_;
          z += coef;
        } else {
          coef = A * wk * rp.k_corr_scale;
        }
        const uint8_t* vr = a.cache.v_codes + (pg * kPage + t) * d.R;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int c = lane + 32 * jj;
          if (c < D) {
            const float svv = read_scale(a.cache.v_scale, (pg * kPage + t) * d.G + c / d.gsize, d.scale_mode, mv);
            const float vh = f16r(__fmul_rn(static_cast<float>(unpack_code(vr, c, d.bits)), svv));
            num[jj] = fmaf(coef, exact ? vh : (vh - sO[i][c]), num[jj]);
          }
        }
      }
    }
    // V slots: A_t * w_t * R_V,t
    for (int k = 0; k < nsel[i]; ++k) {
      const int e = sel[i][k];
      if (e < KG) continue;
      ++reads_v;
      const int ev = e - KG;
      const int p = ev / d.SV, j = ev % d.SV;
      const int64_t pg = lhp * d.P + p;
      const int vb = a.cache.v_slot_block[pg * d.SV + j];
      const int nv = a.cache.valid[pg];
      const int t0 = vb * d.vtb, t1 = min(t0 + d.vtb, nv);
      const uint8_t* pay = a.cache.v_slot_data + (pg * d.SV + j) * d.vslot_bytes;
      const float rs = f16_bits_to_f32(a.cache.v_slot_scale[pg * d.SV + j]);
      int slot = -1;
      for (int u = 0; u < nkp; ++u) if (kp_sm[i][u] == p) slot = u;
      for (int t = t0; t < t1; ++t) {
        const float A = __fdiv_rn(expf(Sb[i * sstride + p * kPage + t] - sM[i]), sL[i]);
        float w = 1.f;
        if (exact) {
          const float dsv = slot >= 0 ? __fdiv_rn(ds_sm[i][slot][t], a.sqrt_d) : 0.f;
          w = dsv <= 80.f ? cbase * expf(dsv) : expf(dsv - mshift);
        }
        const float coef = A * w;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int c = lane + 32 * jj;
          if (c < D) num[jj] = fmaf(coef, unpack_nibble(pay, (t - t0) * D + c, rs), num[jj]);
        }
      }
    }
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int c = lane + 32 * jj;
      if (c < D) {
        const float ob = sO[i][c];
        const float delta = exact ? (__fdiv_rn(num[jj], z) - ob) : num[jj];
        store_act(a.out, (static_cast<int64_t>(s) * Hq + h * QN + i) * D + c, ob + delta, a.dt);
      }
    }
  }
  if (a.cache.read_counter != nullptr && lane == 0) {
    if (any_k && reads_k) atomicAdd(a.cache.read_counter + (static_cast<int64_t>(a.layer) * d.H + h) * 2, (unsigned long long)reads_k);
    if (reads_v) atomicAdd(a.cache.read_counter + (static_cast<int64_t>(a.layer) * d.H + h) * 2 + 1, (unsigned long long)reads_v);
  }
}

// ─────────────────────────── host launch ───────────────────────────
struct SplitPlan {
  int pps, n_splits;
};

inline SplitPlan split_plan(int n_bh, int p_used) {
  SplitPlan sp;
  const int target = 4 * 148;
  int want = (target + n_bh - 1) / max(1, n_bh);
  want = max(1, want);
  int pps = (p_used + want - 1) / want;
  pps = max(pps, 4);
  sp.pps = pps;
  sp.n_splits = max(1, (p_used + pps - 1) / pps);
  return sp;
}

size_t workspace_bytes(const carekv_config_t& c, int seq_count, int p_used) {
  const int qn = c.num_heads / c.num_kv_heads;
  const int64_t n_bh = static_cast<int64_t>(seq_count) * c.num_kv_heads;
  const SplitPlan sp = split_plan(static_cast<int>(n_bh), p_used);
  size_t bytes = 0;
  bytes += n_bh * qn * static_cast<int64_t>(p_used) * kPage * 4;                     // S
  bytes += n_bh * sp.n_splits * qn * 2 * 4;                                          // m, l
  bytes += n_bh * sp.n_splits * qn * static_cast<int64_t>(c.head_dim) * 4;           // O partials
  bytes += n_bh * qn * static_cast<int64_t>(p_used) * (c.k_slots_per_page + c.v_slots_per_page) * 4;
  bytes += n_bh * qn * (kMaxSel + 1) * 4;
  return bytes + 1024;
}

template <int QN>
static cudaError_t launch_qn(DecodeArgs& a, cudaStream_t st, int n_bh) {
  dim3 g1(n_bh, a.n_splits);
  if (a.cfg.head_dim == 64) decode_partial_kernel<QN, 2><<<g1, 128, 0, st>>>(a);
  else decode_partial_kernel<QN, 4><<<g1, 128, 0, st>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  route_kernel<QN><<<n_bh, 256, 0, st>>>(a);
  return cudaGetLastError();
}

int decode_attention(const carekv_config_t& cfg, const carekv_cache_t& cache, int layer, const void* q,
                     void* out, int dtype, int seq_begin, int seq_count, int p_used,
                     const carekv_route_params_t& rp, void* ws, size_t ws_bytes, const float* sketch_proj,
                     cudaStream_t st) {
  if (ws_bytes < workspace_bytes(cfg, seq_count, p_used)) return CAREKV_ERR_WORKSPACE;
  DecodeArgs a;
  a.cfg = cfg;
  a.cache = cache;
  a.layer = layer;
  a.q = q;
  a.out = out;
  a.dt = dtype;
  a.seq_begin = seq_begin;
  a.qn = cfg.num_heads / cfg.num_kv_heads;
  const int n_bh = seq_count * cfg.num_kv_heads;
  const SplitPlan sp = split_plan(n_bh, p_used);
  a.pps = sp.pps;
  a.n_splits = sp.n_splits;
  a.p_used = p_used;
  a.sf = static_cast<float>(1.0 / std::sqrt(static_cast<double>(cfg.head_dim)));
  a.sqrt_d = static_cast<float>(std::sqrt(static_cast<double>(cfg.head_dim)));
  // workspace: selection readback and scores first (their offsets do not
  // depend on the split plan), then logits and split partials
  char* w = static_cast<char*>(ws);
  const int64_t qn = a.qn;
  a.sel_out = reinterpret_cast<int*>(w);
  w += static_cast<int64_t>(n_bh) * qn * (kMaxSel + 1) * 4;
  a.scores = reinterpret_cast<float*>(w);
  w += static_cast<int64_t>(n_bh) * qn * p_used * (cfg.k_slots_per_page + cfg.v_slots_per_page) * 4;
  a.S = reinterpret_cast<float*>(w);
  w += n_bh * qn * static_cast<int64_t>(p_used) * kPage * 4;
  a.pm = reinterpret_cast<float*>(w);
  w += static_cast<int64_t>(n_bh) * sp.n_splits * qn * 4;
  a.pl = reinterpret_cast<float*>(w);
  w += static_cast<int64_t>(n_bh) * sp.n_splits * qn * 4;
  a.po = reinterpret_cast<float*>(w);
  a.sketch_proj = sketch_proj;
  a.rp = rp;
  cudaError_t e;
  switch (a.qn) {
    case 1: e = launch_qn<1>(a, st, n_bh); break;
    case 2: e = launch_qn<2>(a, st, n_bh); break;
    case 4: e = launch_qn<4>(a, st, n_bh); break;
    case 8: e = launch_qn<8>(a, st, n_bh); break;
    default: return CAREKV_ERR_UNSUPPORTED;
  }
  return e == cudaSuccess ? CAREKV_OK : CAREKV_ERR_CUDA;
}

}  // namespace carekv
