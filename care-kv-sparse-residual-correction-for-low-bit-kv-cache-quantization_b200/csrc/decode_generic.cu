// Generic split-K decode pass (kernel K3) for the layouts the tiled passes
// do not take: fp16 / bf16 / fp32 base scales, INT2, groups narrower than a
// quarter row, and the KIVI base (per-channel K scales over the prefill,
// per-token V scales, fp16 K rows of decode-appended tokens).
//
// Same contract as the tiled passes: logits of every token to the
// workspace, q . R_K of every stored K slot (when live combined_kvscore may
// read it), one (m, l, O) partial per CTA.  K_hat and V_hat are the values
// of the reference's fp16 dequantization (cache.py:713-718, the KIVI side
// buffer cache.py:800-865): code * scale rounded once to fp16 (KIVI: to the
// activation dtype, then fp16).
//
// Layout: a CTA of 4 warps streams a page range of one (sequence, kv head);
// each warp takes a page at a time, copies its packed K / V rows and scales
// into a private shared-memory stage with 16-byte loads (one round trip),
// then
//  * logits: lane (t, half) = (lane & 15, lane >> 4) dots half of token t's
//    K row with every query of the group (queries in shared memory), one
//    shuffle joins the halves;
//  * an online softmax per page (16 tokens at once);
//  * values: lane l accumulates the weighted V_hat of D/32 consecutive
//    channels over the page's tokens;
//  * q . R_K of each stored K slot on the tensor cores (queries on the MMA
//    rows as hi / lo fp16 halves, the slot's 4-bit codes as exact fp16
//    integers, the slot scale applied to the fp32 result).
// Reference: attention.py:979-1039 (base decode), attention.py:167-184
// (q . R_K of combined_kvscore).
#include "common.cuh"
#include "internal.h"
#include "decode_args.h"
#include "ptx.cuh"

namespace carekv {
namespace generic {

constexpr int kWarps = 4;
constexpr int kRowStage = 16 * 64;     // packed rows of one page and kind (D <= 128, INT4)
constexpr int kScaleStage = 16 * 8 * 4;  // scales of one page and kind (G <= 8, fp32)

struct WarpStage {
  __align__(16) uint8_t k[kRowStage];
  __align__(16) uint8_t v[kRowStage];
  __align__(16) uint8_t ks[kScaleStage];
  __align__(16) uint8_t vs[kScaleStage];
};

// n bytes (a multiple of 16, both ends 16-byte aligned) by the warp's lanes
__device__ __forceinline__ void warp_copy16(uint8_t* dst, const uint8_t* src, int n, int lane) {
  for (int i = lane; i < n / 16; i += 32)
    reinterpret_cast<uint4*>(dst)[i] = __ldg(reinterpret_cast<const uint4*>(src) + i);
}

template <int QN, int D>
__global__ void __launch_bounds__(kWarps * 32) decode_generic(DecodeArgs a) {
  constexpr int HC = D / 2;     // K channels per lane (half a row)
  constexpr int CPL = D / 32;   // consecutive V channels per lane
  __shared__ __align__(16) float q_sm[QN][D];
  __shared__ float kcs_sm[D];   // KIVI per-channel K scales
  __shared__ __align__(16) uint32_t qfr[D / 32][2][32][4];
  __shared__ WarpStage stg[kWarps];
  __shared__ float sm_m[kWarps][QN], sm_l[kWarps][QN];
  __shared__ float sm_o[kWarps][QN][D];

  const Dims d = make_dims(a.cfg);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  const int bh = blockIdx.x, split = blockIdx.y;
  const int s = bh / d.H, h = bh % d.H, b = a.seq_begin + s;
  const int64_t lhp = d.lhp(b, a.layer, h);
  const int np = min(a.cache.num_pages[lhp], a.p_used);
  const int p0 = split * a.pps, p1 = min(np, p0 + a.pps);
  const int Hq = a.act_heads;   // query heads per activation row
  const int R = d.R, G = d.G;
  const bool kslot = a.kw != nullptr;

  for (int x = threadIdx.x; x < QN * D; x += blockDim.x)
    q_sm[x / D][x % D] = load_act(a.q, (static_cast<int64_t>(s) * Hq + h * QN) * D + x, a.dt);
  int pf = 0;
  if (d.kivi) {
    for (int c = threadIdx.x; c < D; c += blockDim.x) kcs_sm[c] = a.cache.k_chan_scale[lhp * D + c];
    pf = a.cache.prefill_tokens[lhp];
  }
  if (kslot) {
    // A fragments of the slot dots: rows gid = q_hi, gid+8 = q_lo of query
    // gid; k-step ks of group g covers channels g*32 + 8*tig + 4*ks + {0..3}
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
  }
  __syncthreads();

  float m[QN], l[QN], o[QN][CPL];
#pragma unroll
  for (int i = 0; i < QN; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int j = 0; j < CPL; ++j) o[i][j] = 0.f;
  }
  const int t = lane & 15, half = lane >> 4;
  const int ck0 = half * HC;        // the lane's K channels
  const int cv0 = lane * CPL;       // the lane's V channels
  const int64_t sst = static_cast<int64_t>(a.p_used) * kPage;
  float* Srow = a.S + static_cast<int64_t>(bh) * QN * sst;
  const int KG = a.p_used * d.SK;
  float* Wrow = kslot ? a.kw + static_cast<int64_t>(bh) * QN * KG * kPage : nullptr;
  WarpStage& w = stg[warp];
  const int sb = kPage * G * d.scale_elem;   // scale bytes of a page and kind

  for (int p = p0 + warp; p < p1; p += kWarps) {
    const int64_t pg = lhp * d.P + p;
    const int nv = a.cache.valid[pg];
    float mk = 0.f, mv = 0.f;
    if (d.scale_mode == CAREKV_SCALE_INT8) {
      mk = f16_bits_to_f32(a.cache.k_master[pg]);
      mv = f16_bits_to_f32(a.cache.v_master[pg]);
    }
    __syncwarp();   // the previous page's stage is consumed
    warp_copy16(w.k, a.cache.k_codes + pg * kPage * R, kPage * R, lane);
    warp_copy16(w.v, a.cache.v_codes + pg * kPage * R, kPage * R, lane);
    if (!d.kivi) warp_copy16(w.ks, reinterpret_cast<const uint8_t*>(a.cache.k_scale) + pg * sb, sb, lane);
    warp_copy16(w.vs, reinterpret_cast<const uint8_t*>(a.cache.v_scale) + pg * sb, sb, lane);
    __syncwarp();

    // ── logits: lane (t, half) over channels ck0 .. ck0 + HC - 1 ──
    float acc[QN];
#pragma unroll
    for (int i = 0; i < QN; ++i) acc[i] = 0.f;
    if (t < nv) {
      const uint8_t* kr = w.k + t * R;
      const bool packed_row = !d.kivi || p * kPage + t < pf;
      const uint16_t* wrow = packed_row ? nullptr
                                        : a.cache.k_window + ((lhp * d.W + (p - pf / kPage)) * kPage + t) * D;
#pragma unroll 8
      for (int cc = 0; cc < HC; ++cc) {
        const int c = ck0 + cc;
        float kh;
        if (!packed_row) {
          kh = f16_bits_to_f32(wrow[c]);
        } else if (d.kivi) {
          kh = f16r(kivi_hat(unpack_code(kr, c, d.bits), kcs_sm[c], a.dt));
        } else {
          const float sk = read_scale(w.ks, t * G + c / d.gsize, d.scale_mode, mk);
          kh = f16r(__fmul_rn(static_cast<float>(unpack_code(kr, c, d.bits)), sk));
        }
#pragma unroll
        for (int i = 0; i < QN; ++i) acc[i] = fmaf(kh, q_sm[i][c], acc[i]);
      }
    }
    float sv[QN];
#pragma unroll
    for (int i = 0; i < QN; ++i) sv[i] = __fmul_rn(acc[i] + __shfl_xor_sync(0xffffffffu, acc[i], 16), a.sf);
    if (half == 0 && t < nv)
#pragma unroll
      for (int i = 0; i < QN; ++i) Srow[i * sst + p * kPage + t] = sv[i];

    // ── online softmax over the page's tokens, per query ──
    float pr[QN];
#pragma unroll
    for (int i = 0; i < QN; ++i) {
      float pm = t < nv ? sv[i] : -INFINITY;
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, off));
      const float mn = fmaxf(m[i], pm);
      const float corr = m[i] == -INFINITY ? 0.f : expf(m[i] - mn);
      pr[i] = t < nv ? expf(sv[i] - mn) : 0.f;
      float ps = pr[i];
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
      l[i] = l[i] * corr + ps;
#pragma unroll
      for (int j = 0; j < CPL; ++j) o[i][j] *= corr;
      m[i] = mn;
    }

    // ── values: lane over channels cv0 .. cv0 + CPL - 1 ──
    for (int tt = 0; tt < nv; ++tt) {
      const uint8_t* vr = w.v + tt * R;
      float vs_tok = 0.f;
      if (d.kivi) vs_tok = reinterpret_cast<const float*>(w.vs)[tt * G];
      float vh[CPL];
#pragma unroll
      for (int j = 0; j < CPL; ++j) {
        const int c = cv0 + j;
        const int cv = unpack_code(vr, c, d.bits);
        vh[j] = d.kivi ? f16r(kivi_hat(cv, vs_tok, a.dt))
                       : f16r(__fmul_rn(static_cast<float>(cv), read_scale(w.vs, tt * G + c / d.gsize, d.scale_mode, mv)));
      }
#pragma unroll
      for (int i = 0; i < QN; ++i) {
        const float pt = __shfl_sync(0xffffffffu, pr[i], tt);
#pragma unroll
        for (int j = 0; j < CPL; ++j) o[i][j] = fmaf(pt, vh[j], o[i][j]);
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
          float* wr = Wrow + ((static_cast<int64_t>(gid) * KG) + static_cast<int64_t>(p) * d.SK + j) * kPage;
          *reinterpret_cast<float2*>(wr + 2 * tig) =
              make_float2(__fmul_rn(c0[0] + c0[2], rs), __fmul_rn(c0[1] + c0[3], rs));
          *reinterpret_cast<float2*>(wr + 8 + 2 * tig) =
              make_float2(__fmul_rn(c1[0] + c1[2], rs), __fmul_rn(c1[1] + c1[3], rs));
        }
      }
    }
  }

  // ── merge the 4 warps ──
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < QN; ++i) {
      sm_m[warp][i] = m[i];
      sm_l[warp][i] = l[i];
    }
  }
#pragma unroll
  for (int i = 0; i < QN; ++i)
#pragma unroll
    for (int j = 0; j < CPL; ++j) sm_o[warp][i][cv0 + j] = o[i][j];
  __syncthreads();
  const int64_t part = static_cast<int64_t>(bh) * a.n_splits + split;
  for (int idx = threadIdx.x; idx < QN * D; idx += blockDim.x) {
    const int i = idx / D, c = idx % D;
    float M = -INFINITY;
    for (int ww = 0; ww < kWarps; ++ww) M = fmaxf(M, sm_m[ww][i]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
      for (int ww = 0; ww < kWarps; ++ww) {
        const float f = sm_m[ww][i] == -INFINITY ? 0.f : expf(sm_m[ww][i] - M);
        L += sm_l[ww][i] * f;
        O += sm_o[ww][i][c] * f;
      }
    }
    a.po[(part * QN + i) * D + c] = O;
    if (c == 0) {
      a.pm[part * QN + i] = M;
      a.pl[part * QN + i] = L;
    }
  }
}

}  // namespace generic

template <int QN>
cudaError_t launch_decode_generic(DecodeArgs& a, cudaStream_t st, int n_bh) {
  dim3 g(n_bh, a.n_splits);
  if (a.cfg.head_dim == 64) generic::decode_generic<QN, 64><<<g, generic::kWarps * 32, 0, st>>>(a);
  else generic::decode_generic<QN, 128><<<g, generic::kWarps * 32, 0, st>>>(a);
  return cudaGetLastError();
}

template cudaError_t launch_decode_generic<1>(DecodeArgs&, cudaStream_t, int);
template cudaError_t launch_decode_generic<2>(DecodeArgs&, cudaStream_t, int);
template cudaError_t launch_decode_generic<4>(DecodeArgs&, cudaStream_t, int);
template cudaError_t launch_decode_generic<8>(DecodeArgs&, cudaStream_t, int);

}  // namespace carekv
