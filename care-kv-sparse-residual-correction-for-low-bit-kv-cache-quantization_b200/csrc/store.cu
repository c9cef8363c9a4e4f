// Quantize-and-pack on append plus per-page residual enumeration and slot
// storage (kernel K1).
//
// Replaces, for the uniform per-group base:
//   layer.py:204-334      _write_pages_for_kv_head (prefill pages)
//   layer.py:1028-1146    decode append and the page-full re-store
//   cache.py:592-701      write_base / append_to_page / int8 page scales
//   residual_store.py:239-464  ResidualStoreManager.process_page
//
// One CTA processes one 16-row page of one (sequence, kv head): rows are
// staged in shared memory, quantized per group, packed into the reference's
// row format, the page's int8 scale codes and fp16 master are written, the
// residual R = X - X_hat is formed in place, and one warp per candidate
// (K channel group or V token block) computes its error norm, sketch and
// 4-bit payload.  Thread 0 then ranks the candidates and writes the kept
// slots in ascending group order.  Slot ids that reproduce the reference's
// sequential arena allocation are assigned afterwards by a per-sequence scan
// in (kv head, page) order.
#include "common.cuh"
#include "internal.h"

namespace carekv {

struct StoreSmem {
  // sized for head_dim <= 128, page 16, slot capacity <= 8, 8 candidates
  float x[2][kPage][128];        // K, V rows, then residuals in place
  int8_t code[2][kPage][128];
  float sc[2][kPage][4];         // unquantized group scales (dtype values)
  float rscale[2][kPage][4];     // scales as read back (fp16 values)
  float err[8];
  float s4[8];                   // fp32 4-bit slot scale per candidate
  union {
    __align__(16) uint8_t packed[2][kPage * 64];  // packed K / V rows before their store
    __align__(16) uint8_t payload[8][256];        // 4-bit payload per candidate
  };
  float red[2][32];
  float master[2];
  int keep_k[8], keep_v[8];      // kept candidates in slot order
};

constexpr int kStoreThreads = 256;

// 16-byte copy of n bytes (n a multiple of 16, both ends 16-byte aligned)
// by the CTA's threads, else a byte loop.
__device__ __forceinline__ void cta_copy(uint8_t* dst, const uint8_t* src, int n, bool vec) {
  if (vec) {
    for (int i = threadIdx.x; i < n / 16; i += blockDim.x)
      reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
  } else {
    for (int i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
  }
}
__device__ __forceinline__ bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Page store.  mode 0: rows come from K/V inputs (prefill).  mode 1: rows are
// rebuilt from the cache's last page (decode page-full store, layer.py:1087-1146).
template <int MODE>
__global__ void __launch_bounds__(256) page_store_kernel(
    carekv_config_t cfg, carekv_cache_t cache, int layer, const void* __restrict__ Kin,
    const void* __restrict__ Vin, int T, int seq_begin, carekv_store_params_t prm, int in_H,
    const float* __restrict__ sketch_proj) {
  __shared__ StoreSmem sm;
  const Dims d = make_dims_p2(cfg);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int h = blockIdx.y;
  const int s = blockIdx.z;
  const int b = seq_begin + s;
  const int dt = prm.input_dtype;
  const int D = d.D;
  const int64_t lhp = d.lhp(b, layer, h);
  // D (64 / 128), the group size, G and the V token block are powers of two
  // (cache init checks the first and the others divide them), so index
  // arithmetic below uses shifts
  const int lgD = __ffs(D) - 1, lgGs = __ffs(d.gsize) - 1, lgG = __ffs(d.G) - 1;

  int p, nv;
  if (MODE == 0) {
    const int np0 = cache.num_pages[lhp];
    p = np0 + blockIdx.x;
    const int t0 = blockIdx.x * kPage;
    nv = min(kPage, T - t0);
    if (p >= d.P) {
      if (tid == 0) atomicOr(cache.error_flag, kErrPageOverflow);
      return;
    }
    // stage rows; padded rows are zero (layer.py:262-271)
    const int64_t base = ((static_cast<int64_t>(s) * in_H + h) * T + t0) * D;
    const int esz = dt == CAREKV_F32 ? 4 : 2;
    if (al16(Kin) && al16(Vin) && (D * esz) % 16 == 0 && blockDim.x == kStoreThreads) {
      // 16-byte chunks of both pages (at most 4 per thread for D <= 128),
      // every load issued before the first conversion
      const int lgP = esz == 4 ? 2 : 3, per = 1 << lgP, nchunk = (kPage * D) >> lgP, lgN = __ffs(nchunk) - 1;
      uint4 ld[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = tid + u * kStoreThreads;
        ld[u] = make_uint4(0u, 0u, 0u, 0u);
        if (i < 2 * nchunk) {
          const int e0 = (i & (nchunk - 1)) * per;
          if ((e0 >> lgD) < nv)
            ld[u] = *reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(i < nchunk ? Kin : Vin) +
                                                    (base + e0) * esz);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = tid + u * kStoreThreads;
        if (i < 2 * nchunk) {
          const int kind = i >> lgN, e0 = (i & (nchunk - 1)) * per;
          float* dst = &sm.x[kind][e0 >> lgD][e0 & (D - 1)];
          const uint32_t w[4] = {ld[u].x, ld[u].y, ld[u].z, ld[u].w};
          if (esz == 4) {
#pragma unroll
            for (int k = 0; k < 4; ++k) dst[k] = __uint_as_float(w[k]);
          } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint16_t lo = static_cast<uint16_t>(w[k]), hi = static_cast<uint16_t>(w[k] >> 16);
              dst[2 * k] = dt == CAREKV_F16 ? f16_bits_to_f32(lo) : __bfloat162float(__ushort_as_bfloat16(lo));
              dst[2 * k + 1] = dt == CAREKV_F16 ? f16_bits_to_f32(hi) : __bfloat162float(__ushort_as_bfloat16(hi));
            }
          }
        }
      }
    } else {
      for (int i = tid; i < kPage * D; i += blockDim.x) {
        const int r = i >> lgD, c = i & (D - 1);
        float kv = 0.f, vv = 0.f;
        if (r < nv) {
          kv = load_act(Kin, base + static_cast<int64_t>(r) * D + c, dt);
          vv = load_act(Vin, base + static_cast<int64_t>(r) * D + c, dt);
        }
        sm.x[0][r][c] = kv;
        sm.x[1][r][c] = vv;
      }
    }
  } else {
    p = cache.num_pages[lhp] - 1;
    if (p < 0) return;
    const int64_t pg = lhp * d.P + p;
    if (cache.valid[pg] != kPage) return;  // only the page this step filled
    nv = kPage;
    if (d.kivi) {
      // KIVI: the reference re-stores a page filled by decode with K_orig :=
      // K_hat and V_orig := V_hat from its fp16 side buffer (layer.py:1089-1101):
      // every residual is exactly 0
      for (int i = tid; i < kPage * D; i += blockDim.x) {
        sm.x[0][i >> lgD][i & (D - 1)] = 0.f;
        sm.x[1][i >> lgD][i & (D - 1)] = 0.f;
      }
    }
    const float mk = cfg.scale_mode == CAREKV_SCALE_INT8 ? f16_bits_to_f32(cache.k_master[pg]) : 0.f;
    const float mv = cfg.scale_mode == CAREKV_SCALE_INT8 ? f16_bits_to_f32(cache.v_master[pg]) : 0.f;
    for (int i = tid; i < (d.kivi ? 0 : kPage * D); i += blockDim.x) {
      const int r = i >> lgD, c = i & (D - 1);
      const int64_t srow = (pg * kPage + r) * d.G + (c >> lgGs);
      const float sk = read_scale(cache.k_scale, srow, d.scale_mode, mk);
      const float sv = read_scale(cache.v_scale, srow, d.scale_mode, mv);
      const int ck = unpack_code(cache.k_codes + (pg * kPage + r) * d.R, c, d.bits);
      const int cv = unpack_code(cache.v_codes + (pg * kPage + r) * d.R, c, d.bits);
      // K_hat in fp16 (scales are read back as fp16), K_orig := K_hat cast to
      // the model dtype; R = K_orig - K_hat in the promoted dtype.
      const float kh = f16r(__fmul_rn(static_cast<float>(ck), sk));
      const float vh = f16r(__fmul_rn(static_cast<float>(cv), sv));
      sm.x[0][r][c] = rnd(kh, dt) - kh;  // exact: both fp32-representable
      sm.x[1][r][c] = rnd(vh, dt) - vh;
      // fp16 model dtype: promoted dtype is fp16 and rnd() is exact -> 0
    }
  }
  __syncthreads();

  const int64_t pg = lhp * d.P + p;
  const int qmax = (1 << (d.bits - 1)) - 1;

  if (MODE == 0) {
    // ── per-group quantization (quantizer.py:31-64) ──
    const int gs = d.gsize;
    if (d.kivi) {
      // KIVI (kivi_helpers.py:35-59): K codes with the per-channel scale of
      // the whole prefill (k_chan_scale), V codes with a per-token scale; the
      // padded rows of a last page are zero with zero scales (the reference
      // pads K_hat / V_hat with zeros after quantizing, layer.py:279-292)
      const float* cs = cache.k_chan_scale + lhp * D;
      for (int r = warp; r < kPage; r += blockDim.x / 32) {
        float m = 0.f;
        for (int c = lane; c < D; c += 32) m = fmaxf(m, fabsf(sm.x[1][r][c]));
        m = warp_max(m);
        const float vs = r < nv ? kivi_scale(m, qmax, dt) : 0.f;
        for (int c = lane; c < D; c += 32) {
          sm.code[1][r][c] = r < nv ? static_cast<int8_t>(kivi_code_dt(sm.x[1][r][c], vs, qmax, dt)) : 0;
          sm.code[0][r][c] = r < nv ? static_cast<int8_t>(kivi_code_dt(sm.x[0][r][c], cs[c], qmax, dt)) : 0;
        }
        if (lane == 0) {
          sm.sc[1][r][0] = vs;
          sm.sc[0][r][0] = 0.f;   // K scales are per channel (k_chan_scale)
        }
      }
    } else if ((D == 64 || D == 128) && (gs == 16 || gs == 32 || gs == 64 || gs == 128) && D % gs == 0) {
      // warp per (kind, row), lane on channels lane + 32k: the group maximum
      // is a segmented (gs = 16) or whole-warp max combined over the
      // group's columns; max is order-free, so the scale is the reference's
      const int KD = D / 32;
      for (int t = warp; t < 2 * kPage; t += blockDim.x / 32) {
        const int kind = t / kPage, r = t % kPage;
        float xv[4], m[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          xv[k] = k < KD ? sm.x[kind][r][lane + 32 * k] : 0.f;
          m[k] = fmaxf(0.f, fabsf(xv[k]));
        }
        if (gs == 16) {
#pragma unroll
          for (int k = 0; k < 4; ++k)
#pragma unroll
            for (int o = 1; o < 16; o <<= 1) m[k] = fmaxf(m[k], __shfl_xor_sync(0xffffffffu, m[k], o));
        } else {
#pragma unroll
          for (int k = 0; k < 4; ++k) m[k] = warp_max(m[k]);
          if (gs >= 64) {
            m[0] = m[1] = fmaxf(m[0], m[1]);
            m[2] = m[3] = fmaxf(m[2], m[3]);
          }
          if (gs == 128) m[0] = m[1] = m[2] = m[3] = fmaxf(m[0], m[2]);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (k < KD) {
            const int c = lane + 32 * k;
            const float scale = group_scale(m[k], qmax, dt);
            sm.code[kind][r][c] = quant_code(xv[k], scale, qmax, dt);
            if ((c & (gs - 1)) == 0) sm.sc[kind][r][c >> lgGs] = scale;
          }
        }
      }
    } else {
      for (int task = tid; task < 2 * kPage * d.G; task += blockDim.x) {
        const int kind = task >> (4 + lgG);
        const int r = (task >> lgG) & (kPage - 1);
        const int g = task & (d.G - 1);
        float mx = 0.f;
        for (int c = g * d.gsize; c < (g + 1) * d.gsize; ++c) mx = fmaxf(mx, fabsf(sm.x[kind][r][c]));
        const float scale = group_scale(mx, qmax, dt);
        sm.sc[kind][r][g] = scale;
        for (int c = g * d.gsize; c < (g + 1) * d.gsize; ++c)
          sm.code[kind][r][c] = quant_code(sm.x[kind][r][c], scale, qmax, dt);
      }
    }
    __syncthreads();
    // ── packed rows, all 16 rows (cache.py:636-640), staged then stored ──
    const int R = d.R;
    if (d.bits == 3) {
      const int WPR = D / 8, lgW = lgD - 3;   // 24-bit words (8 codes) per row
      for (int i = tid; i < 2 * kPage * WPR; i += blockDim.x) {
        const int kind = i >> (4 + lgW), r = (i >> lgW) & (kPage - 1), w = i & (WPR - 1);
        const int8_t* cp = &sm.code[kind][r][8 * w];
        uint32_t word = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) word |= (static_cast<uint32_t>(cp[k]) & 7u) << (3 * k);
        uint8_t* dst = &sm.packed[kind][r * R + 3 * w];
        dst[0] = static_cast<uint8_t>(word);
        dst[1] = static_cast<uint8_t>(word >> 8);
        dst[2] = static_cast<uint8_t>(word >> 16);
      }
    } else {
      const int lgR = __ffs(R) - 1;   // D/4 or D/2 bytes
      for (int i = tid; i < 2 * kPage * R; i += blockDim.x) {
        const int kind = i >> (4 + lgR), r = (i >> lgR) & (kPage - 1), j = i & (R - 1);
        sm.packed[kind][r * R + j] = pack_byte(&sm.code[kind][r][0], j, d.bits);
      }
    }
    __syncthreads();
    {
      uint8_t* kd = cache.k_codes + pg * kPage * R;
      uint8_t* vd = cache.v_codes + pg * kPage * R;
      const bool vec = (kPage * R) % 16 == 0 && al16(kd) && al16(vd);
      cta_copy(kd, sm.packed[0], kPage * R, vec);
      cta_copy(vd, sm.packed[1], kPage * R, vec);
    }
    // ── page scales (cache.py:592-606) ──
    if (d.scale_mode == CAREKV_SCALE_INT8) {
      for (int kind = 0; kind < 2; ++kind) {
        float mx = 0.f;
        for (int i = tid; i < kPage * d.G; i += blockDim.x) mx = fmaxf(mx, fabsf(sm.sc[kind][i >> lgG][i & (d.G - 1)]));
        mx = warp_max(mx);
        if (lane == 0) sm.red[kind][warp] = mx;
      }
      __syncthreads();
      if (tid < 2) {
        float mx = 0.f;
        for (int w = 0; w < static_cast<int>(blockDim.x / 32); ++w) mx = fmaxf(mx, sm.red[tid][w]);
        mx = fmaxf(mx, clamp_lo(dt));
        const uint16_t mb = f32_to_f16_bits(__fdiv_rn(mx, 127.0f));
        (tid == 0 ? cache.k_master : cache.v_master)[pg] = mb;
        sm.master[tid] = f16_bits_to_f32(mb);
      }
      __syncthreads();
      for (int i = tid; i < 2 * kPage * d.G; i += blockDim.x) {
        const int kind = i >> (4 + lgG);
        const int r = (i >> lgG) & (kPage - 1), g = i & (d.G - 1);
        const int8_t c8 = int8_scale_code(sm.sc[kind][r][g], sm.master[kind]);
        reinterpret_cast<int8_t*>(kind == 0 ? cache.k_scale : cache.v_scale)[(pg * kPage + r) * d.G + g] = c8;
        sm.rscale[kind][r][g] = f16r(__fmul_rn(static_cast<float>(c8), sm.master[kind]));
      }
    } else {
      for (int i = tid; i < 2 * kPage * d.G; i += blockDim.x) {
        const int kind = i >> (4 + lgG);
        const int r = (i >> lgG) & (kPage - 1), g = i & (d.G - 1);
        void* dst = kind == 0 ? cache.k_scale : cache.v_scale;
        const int64_t idx = (pg * kPage + r) * d.G + g;
        write_raw_scale(dst, idx, d.scale_mode, sm.sc[kind][r][g]);
        sm.rscale[kind][r][g] = read_scale(dst, idx, d.scale_mode, 0.f);
      }
    }
    if (tid == 0) cache.valid[pg] = nv;
    __syncthreads();
    // ── residual in place (residual_store.py:271-285) + V_hat norm ──
    float vn = 0.f;
    const float* kcs = d.kivi ? cache.k_chan_scale + lhp * D : nullptr;
    for (int i = tid; i < kPage * D; i += blockDim.x) {
      const int r = i >> lgD, c = i & (D - 1), g = c >> lgGs;
      if (r < nv) {
        const float kh = dequant(sm.code[0][r][c], d.kivi ? kcs[c] : sm.sc[0][r][g], dt);
        const float vh = dequant(sm.code[1][r][c], sm.sc[1][r][g], dt);
        sm.x[0][r][c] = rnd(__fsub_rn(sm.x[0][r][c], kh), dt);
        sm.x[1][r][c] = rnd(__fsub_rn(sm.x[1][r][c], vh), dt);
        // the V rows as stored: fp16 of V_hat (the KIVI side buffer holds
        // fp16(V_hat)), or code * the scale as read back
        const float vr = d.kivi ? f16r(vh) : f16r(__fmul_rn(static_cast<float>(sm.code[1][r][c]), sm.rscale[1][r][g]));
        vn = fmaf(vr, vr, vn);
      } else {
        sm.x[0][r][c] = 0.f;
        sm.x[1][r][c] = 0.f;
      }
    }
    vn = warp_sum(vn);
    if (lane == 0) sm.red[0][warp] = vn;
    __syncthreads();
    if (tid == 0) {
      float t = 0.f;
      for (int w = 0; w < static_cast<int>(blockDim.x / 32); ++w) t += sm.red[0][w];
      cache.v_norm2[pg] = t;
    }
  }
  __syncthreads();

  // ── candidates: warp w < C -> K channel group, then V token blocks ──
  const int ncand = d.C + d.NV;
  for (int cand = warp; cand < ncand; cand += blockDim.x / 32) {
    if (cand < d.C) {
      const int c0 = cand * d.kcg;  // kcg == 32: lane = channel
      float err = 0.f, colsum = 0.f, mx = 0.f;
      for (int r = 0; r < kPage; ++r) {
        const float v = sm.x[0][r][c0 + lane];
        mx = fmaxf(mx, fabsf(v));
        if (r < nv) {
          const float n = sqrtf(warp_sum(v * v));
          err += n;
          colsum += v;
        }
      }
      mx = warp_max(mx);
      if (lane == 0) sm.err[cand] = nv > 0 ? __fdiv_rn(err, static_cast<float>(nv)) : 0.f;
      const float sc4 = __fdiv_rn(fmaxf(mx, 1e-8f), 7.0f);
      if (lane == 0) sm.s4[cand] = sc4;
      // payload: value index i = t*32 + c, byte i/2 (residual_store.py:127-136)
      for (int j = lane; j < d.kslot_bytes; j += 32) {
        const int i0 = 2 * j;
        const int t = i0 >> 5, c = i0 & 31;   // kcg == 32
        const int lo = nibble_code(sm.x[0][t][c0 + c], sc4);
        const int hi = nibble_code(sm.x[0][t][c0 + c + 1], sc4);
        sm.payload[cand][j] = static_cast<uint8_t>((lo & 15) | ((hi & 15) << 4));
      }
      // sketch = fp16(mean_t R @ P) (residual_store.py:302-312)
      if (cache.k_sketch != nullptr && d.sketch > 0) {
        const float mean = nv > 0 ? __fdiv_rn(colsum, static_cast<float>(nv)) : 0.f;
        for (int jj = 0; jj < d.sketch; jj += 32) {
          const int j = jj + lane;
          float acc = 0.f;
          for (int c = 0; c < d.kcg; ++c) {
            const float mc = __shfl_sync(0xffffffffu, mean, c);
            if (j < d.sketch) acc = fmaf(mc, sketch_proj[c * d.sketch + j], acc);
          }
          if (j < d.sketch)
            cache.k_sketch[(pg * d.C + cand) * d.sketch + j] = f32_to_f16_bits(acc);
        }
      }
    } else {
      const int vb = cand - d.C;
      const int t0 = vb * d.vtb;
      float err = 0.f, mx = 0.f;
      for (int r = t0; r < t0 + d.vtb; ++r) {
        float ss = 0.f;
        for (int c = lane; c < D; c += 32) {
          const float v = sm.x[1][r][c];
          ss = fmaf(v, v, ss);
          mx = fmaxf(mx, fabsf(v));
        }
        if (r < nv) err += sqrtf(warp_sum(ss));
      }
      mx = warp_max(mx);
      const int t1 = min(t0 + d.vtb, nv);
      if (lane == 0) sm.err[cand] = t1 > t0 ? __fdiv_rn(err, static_cast<float>(t1 - t0)) : 0.f;
      const float sc4 = __fdiv_rn(fmaxf(mx, 1e-8f), 7.0f);
      if (lane == 0) sm.s4[cand] = sc4;
      for (int j = lane; j < d.vslot_bytes; j += 32) {
        const int i0 = 2 * j;
        const int t = t0 + (i0 >> lgD), c = i0 & (D - 1);
        const int lo = nibble_code(sm.x[1][t][c], sc4);
        const int hi = nibble_code(sm.x[1][t][c + 1], sc4);
        sm.payload[cand][j] = static_cast<uint8_t>((lo & 15) | ((hi & 15) << 4));
      }
    }
  }
  __syncthreads();

  // ── selection (residual_store.py:370-423) and slot tables ──
  // Warp 0, lane x = candidate x (K channel groups, then V token blocks).
  // The reference sorts each kind stably by descending error (positive
  // errors only), merges the two lists stably (K first on equal errors),
  // keeps the first joint_budget (or k_budget / v_budget), caps them at the
  // slot capacity and stores the kept ones in ascending group order with
  // their sorted rank as slot id.  Here every lane computes its own rank
  // and merged position by counting, so no thread sorts.
  if (warp == 0) {
    const int ncand = d.C + d.NV;
    const bool pos = prm.sensitivity > 0.f && !prm.store_nothing;
    const bool isk = lane < d.C, isv = lane >= d.C && lane < ncand;
    const float e = (isk || isv) ? sm.err[lane] : 0.f;
    const bool elig = (isk || isv) && pos && e > 0.f;
    int rank = 0, other = 0;   // rank in its kind; merged-order predecessors of the other kind
    for (int o = 0; o < ncand; ++o) {
      const float eo = sm.err[o];
      if (!(pos && eo > 0.f)) continue;
      if ((o < d.C) == isk) {
        if (eo > e || (eo == e && o < lane)) ++rank;
      } else {
        if (isk ? eo > e : eo >= e) ++other;   // a V entry precedes a K entry only with a larger error
      }
    }
    const unsigned bk = __ballot_sync(0xffffffffu, elig && isk), bv = __ballot_sync(0xffffffffu, elig && isv);
    const int n_k = __popc(bk), n_v = __popc(bv);
    int keep_k, keep_v;
    if (prm.joint_budget > 0) {
      const bool in = elig && rank + other < prm.joint_budget;
      keep_k = __popc(__ballot_sync(0xffffffffu, in && isk));
      keep_v = __popc(__ballot_sync(0xffffffffu, in && isv));
    } else {
      keep_k = min(n_k, prm.k_budget);
      keep_v = min(n_v, prm.v_budget);
    }
    keep_k = min(keep_k, d.SK);
    keep_v = min(keep_v, d.SV);
    const bool kept_k = elig && isk && rank < keep_k, kept_v = elig && isv && rank < keep_v;
    const unsigned mk = __ballot_sync(0xffffffffu, kept_k), mv = __ballot_sync(0xffffffffu, kept_v);
    const unsigned lt = (1u << lane) - 1u;
    const int nk = __popc(mk), nvk = __popc(mv);
    if (kept_k) {
      const int j = __popc(mk & lt);
      const int64_t sidx = pg * d.SK + j;
      cache.k_slot_group[sidx] = static_cast<int8_t>(lane);
      cache.k_slot_scale[sidx] = f32_to_f16_bits(sm.s4[lane]);
      cache.k_slot_id[sidx] = rank;  // local rank; the scan adds the arena base
      sm.keep_k[j] = lane;
    }
    if (kept_v) {
      const int j = __popc(mv & lt);
      const int64_t sidx = pg * d.SV + j;
      cache.v_slot_block[sidx] = static_cast<int8_t>(lane - d.C);
      cache.v_slot_scale[sidx] = f32_to_f16_bits(sm.s4[lane]);
      cache.v_slot_id[sidx] = rank;
      sm.keep_v[j] = lane - d.C;
    }
    if (lane >= nk && lane < d.SK) {
      cache.k_slot_group[pg * d.SK + lane] = -1;
      cache.k_slot_id[pg * d.SK + lane] = -1;
    }
    if (lane >= nvk && lane < d.SV) {
      cache.v_slot_block[pg * d.SV + lane] = -1;
      cache.v_slot_id[pg * d.SV + lane] = -1;
    }
    if (isk) cache.k_err[pg * d.C + lane] = f32_to_f16_bits(e);
    if (isv) cache.v_err[pg * d.NV + lane - d.C] = f32_to_f16_bits(e);
    if (lane == 0) {
      sm.red[1][0] = __int_as_float(nk);
      sm.red[1][1] = __int_as_float(nvk);
    }
  }
  __syncthreads();
  // payload copies of the kept slots
  const int nk = __float_as_int(sm.red[1][0]);
  const int nvk = __float_as_int(sm.red[1][1]);
  for (int j = 0; j < nk; ++j) {
    uint8_t* dst = cache.k_slot_data + (pg * d.SK + j) * d.kslot_bytes;
    cta_copy(dst, sm.payload[sm.keep_k[j]], d.kslot_bytes, d.kslot_bytes % 16 == 0 && al16(dst));
  }
  for (int j = 0; j < nvk; ++j) {
    uint8_t* dst = cache.v_slot_data + (pg * d.SV + j) * d.vslot_bytes;
    cta_copy(dst, sm.payload[d.C + sm.keep_v[j]], d.vslot_bytes, d.vslot_bytes % 16 == 0 && al16(dst));
  }
}

// Assign reference arena ids: pages of this call in (kv head, page) order,
// K and V counted separately; then advance the per-sequence counters and,
// for prefill, the page counts.  One CTA per sequence.
// MODE 0: pages [np0, np0+n_new) per head (prefill).  MODE 1: the last page
// of each head when it is full (decode page-full store).
template <int MODE>
__global__ void __launch_bounds__(1024) slot_id_scan_kernel(carekv_config_t cfg, carekv_cache_t cache,
                                                            int layer, int seq_begin, int n_new) {
  const Dims d = make_dims(cfg);
  const int b = seq_begin + blockIdx.x;
  const int tid = threadIdx.x;
  const int npg = (MODE == 0) ? n_new : 1;
  const int total = d.H * npg;
  __shared__ int sk[1024], sv[1024];
  __shared__ int basek, basev;
  if (tid == 0) {
    basek = cache.slot_counter[2 * b];
    basev = cache.slot_counter[2 * b + 1];
  }
  __syncthreads();
  // each thread owns a contiguous chunk of (head, page) entries
  const int per = (total + blockDim.x - 1) / blockDim.x;
  const int lo = tid * per, hi = min(total, lo + per);
  auto page_of = [&](int e, int64_t& pg) -> bool {
    const int h = e / npg, i = e % npg;
    const int64_t lhp = d.lhp(b, layer, h);
    int p;
    if (MODE == 0) {
      p = cache.num_pages[lhp] + i;
      if (p >= d.P) return false;
    } else {
      p = cache.num_pages[lhp] - 1;
      if (p < 0 || cache.valid[lhp * d.P + p] != kPage) return false;
    }
    pg = lhp * d.P + p;
    return true;
  };
  int ck = 0, cv = 0;
  for (int e = lo; e < hi; ++e) {
    int64_t pg;
    if (!page_of(e, pg)) continue;
    for (int j = 0; j < d.SK; ++j) ck += cache.k_slot_group[pg * d.SK + j] >= 0;
    for (int j = 0; j < d.SV; ++j) cv += cache.v_slot_block[pg * d.SV + j] >= 0;
  }
  sk[tid] = ck;
  sv[tid] = cv;
  __syncthreads();
  // inclusive Hillis-Steele scan
  for (int off = 1; off < static_cast<int>(blockDim.x); off <<= 1) {
    const int ak = tid >= off ? sk[tid - off] : 0;
    const int av = tid >= off ? sv[tid - off] : 0;
    __syncthreads();
    sk[tid] += ak;
    sv[tid] += av;
    __syncthreads();
  }
  int ok = basek + sk[tid] - ck, ov = basev + sv[tid] - cv;
  for (int e = lo; e < hi; ++e) {
    int64_t pg;
    if (!page_of(e, pg)) continue;
    int nk = 0, nvv = 0;
    for (int j = 0; j < d.SK; ++j) {
      if (cache.k_slot_group[pg * d.SK + j] >= 0) {
        cache.k_slot_id[pg * d.SK + j] += ok;
        ++nk;
      }
    }
    for (int j = 0; j < d.SV; ++j) {
      if (cache.v_slot_block[pg * d.SV + j] >= 0) {
        cache.v_slot_id[pg * d.SV + j] += ov;
        ++nvv;
      }
    }
    ok += nk;
    ov += nvv;
  }
  __syncthreads();
  if (tid == blockDim.x - 1) {
    cache.slot_counter[2 * b] = basek + sk[tid];
    cache.slot_counter[2 * b + 1] = basev + sv[tid];
  }
  if (MODE == 0) {
    __syncthreads();
    for (int h = tid; h < d.H; h += blockDim.x) {
      const int64_t lhp = d.lhp(b, layer, h);
      cache.num_pages[lhp] = min(d.P, cache.num_pages[lhp] + n_new);
    }
  }
}

// KIVI per-channel K scales of a prefill (quant_dequant_kivi_k over the
// whole prefill, kivi_helpers.py:35-47): first the channel maxima of |K|
// over T, in chunks of rows, folded with an integer max (the bit patterns of
// non-negative floats order like their values) into k_chan_scale, which
// cache init zeroed; then the maxima become scales in place.
constexpr int kKiviRows = 256;   // rows per CTA of the channel maximum
__global__ void __launch_bounds__(128) kivi_chan_amax_kernel(carekv_config_t cfg, carekv_cache_t cache, int layer,
                                                             const void* __restrict__ Kin, int T, int seq_begin,
                                                             int in_H, int dt) {
  const Dims d = make_dims(cfg);
  const int h = blockIdx.y, s = blockIdx.z, b = seq_begin + s;
  const int t0 = blockIdx.x * kKiviRows, t1 = min(T, t0 + kKiviRows);
  const int64_t lhp = d.lhp(b, layer, h);
  const int64_t base = (static_cast<int64_t>(s) * in_H + h) * T * d.D;
  for (int c = threadIdx.x; c < d.D; c += blockDim.x) {
    float m = 0.f;
#pragma unroll 8
    for (int t = t0; t < t1; ++t) m = fmaxf(m, fabsf(load_act(Kin, base + static_cast<int64_t>(t) * d.D + c, dt)));
    atomicMax(reinterpret_cast<unsigned int*>(cache.k_chan_scale + lhp * d.D + c), __float_as_uint(m));
  }
}
__global__ void __launch_bounds__(128) kivi_chan_scale_kernel(carekv_config_t cfg, carekv_cache_t cache, int layer,
                                                              int T, int seq_begin, int dt) {
  const Dims d = make_dims(cfg);
  const int h = blockIdx.x, s = blockIdx.y, b = seq_begin + s;
  const int64_t lhp = d.lhp(b, layer, h);
  const int qmax = (1 << (d.bits - 1)) - 1;
  for (int c = threadIdx.x; c < d.D; c += blockDim.x) {
    float* sc = cache.k_chan_scale + lhp * d.D + c;
    *sc = kivi_scale(*sc, qmax, dt);
  }
  if (threadIdx.x == 0) {
    // the KIVI scales belong to one prefill per (sequence, layer)
    if (cache.num_pages[lhp] != 0 || cache.prefill_tokens[lhp] != 0) atomicOr(cache.error_flag, kErrBadState);
    cache.prefill_tokens[lhp] = T;
  }
}

// Decode append of one row per (sequence, kv head) (layer.py:1028-1085,
// cache.py:656-701).  One warp per (sequence, kv head).
__global__ void __launch_bounds__(32) append_kernel(carekv_config_t cfg, carekv_cache_t cache, int layer,
                                                    const void* __restrict__ kin,
                                                    const void* __restrict__ vin, int seq_begin,
                                                    carekv_store_params_t prm, int in_H) {
  const Dims d = make_dims_p2(cfg);
  const int lane = threadIdx.x;
  const int lgGs = __ffs(d.gsize) - 1, lgG = __ffs(d.G) - 1;   // powers of two (cache init)
  const int h = blockIdx.x, s = blockIdx.y, b = seq_begin + s;
  const int dt = prm.input_dtype;
  const int D = d.D;
  const int64_t lhp = d.lhp(b, layer, h);
  __shared__ float xs[2][128];
  __shared__ int8_t cs[2][128];
  __shared__ float scs[2][4];
  __shared__ int sh_p, sh_off;

  // the new rows first: their loads do not depend on the page state
  const int64_t src = (static_cast<int64_t>(s) * in_H + h) * D;
  for (int c = lane; c < D; c += 32) {
    xs[0][c] = load_act(kin, src + c, dt);
    xs[1][c] = load_act(vin, src + c, dt);
  }
  uint32_t masters = 0;   // lane 0: fp16 K | V master of the target page, read early
  if (lane == 0) {
    const int np = cache.num_pages[lhp];
    int p = np - 1;
    // the last page's fill and masters in one round trip
    int last_valid = kPage;
    if (p >= 0) {
      const int64_t pl = lhp * d.P + p;
      last_valid = cache.valid[pl];
      if (cfg.scale_mode == CAREKV_SCALE_INT8)
        masters = cache.k_master[pl] | (static_cast<uint32_t>(cache.v_master[pl]) << 16);
    }
    if (last_valid >= kPage) {
      masters = 0;
      p = np;
      if (p >= d.P) {
        atomicOr(cache.error_flag, kErrPageOverflow);
        p = -1;
      } else {
        cache.num_pages[lhp] = np + 1;
        const int64_t pg = lhp * d.P + p;
        cache.valid[pg] = 0;
        cache.v_norm2[pg] = 0.f;
        if (cfg.scale_mode == CAREKV_SCALE_INT8) {
          cache.k_master[pg] = 0;  // a decode-opened page keeps master 0 (cache.py:689-695)
          cache.v_master[pg] = 0;
        }
        for (int j = 0; j < d.SK; ++j) { cache.k_slot_group[pg * d.SK + j] = -1; cache.k_slot_id[pg * d.SK + j] = -1; }
        for (int j = 0; j < d.SV; ++j) { cache.v_slot_block[pg * d.SV + j] = -1; cache.v_slot_id[pg * d.SV + j] = -1; }
      }
    }
    sh_p = p;
    sh_off = p == np - 1 ? last_valid : 0;   // a page opened here starts empty
  }
  __syncwarp();
  const int p = sh_p;
  if (p < 0) return;
  const int off = sh_off;
  const int64_t pg = lhp * d.P + p;
  const int qmax = (1 << (d.bits - 1)) - 1;
  if (d.kivi) {
    // KIVI decode append (layer.py:1037-1085): the K row quantized per
    // channel over its single token (scale |k| / qmax per channel), kept as
    // fp16 in the window; the V row quantized per token into the packed page
    const int pf = cache.prefill_tokens[lhp];
    const int wp = p - pf / kPage;   // window page of this page
    if (wp < 0 || wp >= d.W) {
      if (lane == 0) atomicOr(cache.error_flag, kErrPageOverflow);
      return;
    }
    uint16_t* krow = cache.k_window + ((lhp * d.W + wp) * kPage + off) * D;
    float mv = 0.f;
    for (int c = lane; c < D; c += 32) {
      const float x = xs[0][c];
      const float ks = kivi_scale(fabsf(x), qmax, dt);
      krow[c] = f32_to_f16_bits(kivi_hat(kivi_code_dt(x, ks, qmax, dt), ks, dt));
      mv = fmaxf(mv, fabsf(xs[1][c]));
    }
    mv = warp_max(mv);
    const float vs = kivi_scale(mv, qmax, dt);
    for (int c = lane; c < D; c += 32) cs[1][c] = static_cast<int8_t>(kivi_code_dt(xs[1][c], vs, qmax, dt));
    __syncwarp();
    for (int j = lane; j < d.R; j += 32) cache.v_codes[(pg * kPage + off) * d.R + j] = pack_byte(cs[1], j, d.bits);
    if (lane == 0) {
      reinterpret_cast<float*>(cache.v_scale)[pg * kPage + off] = vs;
      reinterpret_cast<float*>(cache.k_scale)[pg * kPage + off] = 0.f;
    }
    float vn = 0.f;
    for (int c = lane; c < D; c += 32) {
      const float vr = f16r(kivi_hat(cs[1][c], vs, dt));
      vn = fmaf(vr, vr, vn);
    }
    vn = warp_sum(vn);
    if (lane == 0) {
      cache.v_norm2[pg] += vn;
      cache.valid[pg] = off + 1;
    }
    return;
  }
  // per-group max |x| of both rows: every lane folds its channels c = lane +
  // 32 t into the (kind, group) maxima, then one butterfly per maximum
  {
    float mx[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int c = lane + 32 * t;
      if (c < D) {
        const int g = c >> lgGs;
#pragma unroll
        for (int gg = 0; gg < 4; ++gg) {
          if (gg == g) {
            mx[0][gg] = fmaxf(mx[0][gg], fabsf(xs[0][c]));
            mx[1][gg] = fmaxf(mx[1][gg], fabsf(xs[1][c]));
          }
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int gg = 0; gg < 4; ++gg) {
        mx[0][gg] = fmaxf(mx[0][gg], __shfl_xor_sync(0xffffffffu, mx[0][gg], o));
        mx[1][gg] = fmaxf(mx[1][gg], __shfl_xor_sync(0xffffffffu, mx[1][gg], o));
      }
    if (lane < 2 * d.G) {
      const int kind = lane >> lgG, g = lane & (d.G - 1);
      float m = mx[0][0];
#pragma unroll
      for (int kk = 0; kk < 2; ++kk)
#pragma unroll
        for (int gg = 0; gg < 4; ++gg)
          if (kk == kind && gg == g) m = mx[kk][gg];
      scs[kind][g] = group_scale(m, qmax, dt);
    }
    __syncwarp();
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int c = lane + 32 * t;
      if (c < D) {
        const int g = c >> lgGs;
        cs[0][c] = quant_code(xs[0][c], scs[0][g], qmax, dt);
        cs[1][c] = quant_code(xs[1][c], scs[1][g], qmax, dt);
      }
    }
  }
  masters = __shfl_sync(0xffffffffu, masters, 0);
  __syncwarp();
  for (int j = lane; j < 2 * d.R; j += 32) {
    const int kind = j >= d.R ? 1 : 0, jj = j - kind * d.R;   // j < 2R
    (kind == 0 ? cache.k_codes : cache.v_codes)[(pg * kPage + off) * d.R + jj] = pack_byte(cs[kind], jj, d.bits);
  }
  __shared__ float rs[2][4];
  if (lane < 2 * d.G) {
    const int kind = lane >> lgG, g = lane & (d.G - 1);
    void* dst = kind == 0 ? cache.k_scale : cache.v_scale;
    const int64_t idx = (pg * kPage + off) * d.G + g;
    if (d.scale_mode == CAREKV_SCALE_INT8) {
      uint16_t mb = static_cast<uint16_t>(kind == 0 ? masters : masters >> 16);
      if (prm.decode_page_master && off == 0 && mb == 0) {
        // a page opened by decode: its first row sets the master the way
        // write_base does for a prefill page (max scale, clamped, / 127)
        float mx = 0.f;
        for (int gg = 0; gg < d.G; ++gg) mx = fmaxf(mx, fabsf(scs[kind][gg]));
        mb = f32_to_f16_bits(__fdiv_rn(fmaxf(mx, clamp_lo(dt)), 127.0f));
        if (g == 0) (kind == 0 ? cache.k_master : cache.v_master)[pg] = mb;
      }
      const float m = f16_bits_to_f32(mb);
      const float mc = fmaxf(m, 1e-8f);  // master.clamp(min=1e-8) in fp32
      const int8_t c8 = int8_scale_code(scs[kind][g], mc);
      reinterpret_cast<int8_t*>(dst)[idx] = c8;
      rs[kind][g] = f16r(__fmul_rn(static_cast<float>(c8), m));
    } else {
      write_raw_scale(dst, idx, d.scale_mode, scs[kind][g]);
      rs[kind][g] = read_scale(dst, idx, d.scale_mode, 0.f);
    }
  }
  __syncwarp();
  float vn = 0.f;
  for (int c = lane; c < D; c += 32) {
    const float vr = f16r(__fmul_rn(static_cast<float>(cs[1][c]), rs[1][c >> lgGs]));
    vn = fmaf(vr, vr, vn);
  }
  vn = warp_sum(vn);
  if (lane == 0) {
    cache.v_norm2[pg] += vn;
    cache.valid[pg] = off + 1;
  }
}

}  // namespace carekv

namespace carekv {

cudaError_t launch_prefill_store(const carekv_config_t& cfg, const carekv_cache_t& cache, int layer, const void* K,
                                 const void* V, int T, int seq_begin, int seq_count,
                                 const carekv_store_params_t& prm, const float* sketch_proj, int in_H,
                                 cudaStream_t st) {
  const int n_new = (T + kPage - 1) / kPage;
  if (n_new == 0 || seq_count == 0) return cudaSuccess;
  if (cfg.base_kind == CAREKV_BASE_KIVI) {
    dim3 ga((T + kKiviRows - 1) / kKiviRows, cfg.num_kv_heads, seq_count);
    kivi_chan_amax_kernel<<<ga, 128, 0, st>>>(cfg, cache, layer, K, T, seq_begin, in_H, prm.input_dtype);
    dim3 gs(cfg.num_kv_heads, seq_count);
    kivi_chan_scale_kernel<<<gs, 128, 0, st>>>(cfg, cache, layer, T, seq_begin, prm.input_dtype);
    cudaError_t e0 = cudaGetLastError();
    if (e0 != cudaSuccess) return e0;
  }
  cudaError_t e;
  if (prefill_store_warp_supported(cfg, cache, K, V, prm)) {
    e = launch_prefill_store_warp(cfg, cache, layer, K, V, T, seq_begin, seq_count, prm, in_H, st);
  } else {
    dim3 grid(n_new, cfg.num_kv_heads, seq_count);
    page_store_kernel<0><<<grid, 256, 0, st>>>(cfg, cache, layer, K, V, T, seq_begin, prm, in_H, sketch_proj);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return e;
  slot_id_scan_kernel<0><<<seq_count, 1024, 0, st>>>(cfg, cache, layer, seq_begin, n_new);
  return cudaGetLastError();
}

cudaError_t launch_append(const carekv_config_t& cfg, const carekv_cache_t& cache, int layer, const void* k,
                          const void* v, int seq_begin, int seq_count, const carekv_store_params_t& prm,
                          const float* sketch_proj, int may_fill, int in_H, cudaStream_t st) {
  if (seq_count == 0) return cudaSuccess;
  dim3 g(cfg.num_kv_heads, seq_count);
  append_kernel<<<g, 32, 0, st>>>(cfg, cache, layer, k, v, seq_begin, prm, in_H);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || !may_fill) return e;
  dim3 g2(1, cfg.num_kv_heads, seq_count);
  page_store_kernel<1><<<g2, 256, 0, st>>>(cfg, cache, layer, nullptr, nullptr, 0, seq_begin, prm, cfg.num_kv_heads,
                                            sketch_proj);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  slot_id_scan_kernel<1><<<seq_count, 1024, 0, st>>>(cfg, cache, layer, seq_begin, 1);
  return cudaGetLastError();
}

}  // namespace carekv
