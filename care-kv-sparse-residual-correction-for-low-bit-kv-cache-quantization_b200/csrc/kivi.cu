// KIVI-style quantize-dequantize (kivi_helpers.py:35-59): symmetric INT
// codes with a per-channel scale over the token axis (K) or a per-token
// scale over the channel axis (V), returned dequantized in the input dtype.
//
// Every step rounds in the input dtype as torch does on the reference's CPU
// path: scale = amax / qmax, clamp(min=1e-8) (0 in fp16), codes =
// clamp(round(x / scale), qmin, qmax) (round half to even; NaN stays NaN),
// out = codes * scale.  amax propagates NaN.
#include "common.cuh"
#include "internal.h"

namespace carekv {
namespace {

__device__ __forceinline__ float nan_max(float a, float b) { return (b != b || b > a) ? b : a; }

__device__ __forceinline__ float kivi_scale(float amax, float qmax, int dt) {
  const float s = rnd(__fdiv_rn(amax, qmax), dt);
  const float lo = clamp_lo(dt);
  return s < lo ? lo : s;  // a NaN scale stays NaN
}

__device__ __forceinline__ float kivi_qdq(float x, float scale, float qmin, float qmax, int dt) {
  float q = rintf(rnd(__fdiv_rn(x, scale), dt));
  if (q == q) q = fminf(fmaxf(q, qmin), qmax);
  return rnd(__fmul_rn(q, scale), dt);
}

// K [n][T][D]: one CTA per (n, 32-channel tile); 8 row groups x 32 channels.
__global__ void __launch_bounds__(256) kivi_k_kernel(const void* __restrict__ x, void* __restrict__ out, int64_t n,
                                                     int T, int D, float qmin, float qmax, int dt) {
  const int tiles = (D + 31) / 32;
  const int64_t nb = blockIdx.x / tiles;
  const int c = (blockIdx.x % tiles) * 32 + (threadIdx.x & 31);
  const int r0 = threadIdx.x >> 5;
  __shared__ float red[8][32];
  const int64_t base = nb * T * static_cast<int64_t>(D);
  float m = 0.f;
  if (c < D)
    for (int t = r0; t < T; t += 8) m = nan_max(m, fabsf(load_act(x, base + static_cast<int64_t>(t) * D + c, dt)));
  red[r0][threadIdx.x & 31] = m;
  __syncthreads();
  float amax = red[0][threadIdx.x & 31];
  for (int r = 1; r < 8; ++r) amax = nan_max(amax, red[r][threadIdx.x & 31]);
  const float sc = kivi_scale(amax, qmax, dt);
  if (c < D)
    for (int t = r0; t < T; t += 8) {
      const int64_t i = base + static_cast<int64_t>(t) * D + c;
      store_act(out, i, kivi_qdq(load_act(x, i, dt), sc, qmin, qmax, dt), dt);
    }
}

// V [rows][D]: one warp per row.
__global__ void __launch_bounds__(256) kivi_v_kernel(const void* __restrict__ x, void* __restrict__ out, int64_t rows,
                                                     int D, float qmin, float qmax, int dt) {
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int64_t base = row * D;
  float m = 0.f;
  for (int c = lane; c < D; c += 32) m = nan_max(m, fabsf(load_act(x, base + c, dt)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = nan_max(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float sc = kivi_scale(m, qmax, dt);
  for (int c = lane; c < D; c += 32) store_act(out, base + c, kivi_qdq(load_act(x, base + c, dt), sc, qmin, qmax, dt), dt);
}

}  // namespace

cudaError_t launch_kivi_k(const void* x, void* out, int64_t n, int T, int D, int bits, int dt, cudaStream_t st) {
  if (n * T * static_cast<int64_t>(D) == 0) return cudaSuccess;
  const float qmax = static_cast<float>((1 << (bits - 1)) - 1), qmin = -static_cast<float>(1 << (bits - 1));
  kivi_k_kernel<<<static_cast<unsigned>(n * ((D + 31) / 32)), 256, 0, st>>>(x, out, n, T, D, qmin, qmax, dt);
  return cudaGetLastError();
}

cudaError_t launch_kivi_v(const void* x, void* out, int64_t rows, int D, int bits, int dt, cudaStream_t st) {
  if (rows * D == 0) return cudaSuccess;
  const float qmax = static_cast<float>((1 << (bits - 1)) - 1), qmin = -static_cast<float>(1 << (bits - 1));
  kivi_v_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, st>>>(x, out, rows, D, qmin, qmax, dt);
  return cudaGetLastError();
}

}  // namespace carekv
