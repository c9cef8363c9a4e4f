// Standalone quantizer ops on contiguous device rows (quantizer.py:31-99,
// 257-383; residual_store.py:121-146).  They back the package's
// quantize / dequantize / pack_codes_2d / pack_4bit functions and share the
// exact device arithmetic of the cache kernels.
#include "common.cuh"
#include "internal.h"

namespace carekv {

// one thread per (row, group)
__global__ void quantize_kernel(const void* __restrict__ x, int8_t* __restrict__ codes, void* __restrict__ scale,
                                int64_t rows, int D, int bits, int gs, int dt) {
  const int G = D / gs;
  const int64_t task = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (task >= rows * G) return;
  const int64_t r = task / G;
  const int g = static_cast<int>(task % G);
  const int qmax = (1 << (bits - 1)) - 1;
  const int64_t base = r * D + static_cast<int64_t>(g) * gs;
  float mx = 0.f;
  for (int c = 0; c < gs; ++c) mx = fmaxf(mx, fabsf(load_act(x, base + c, dt)));
  const float sc = group_scale(mx, qmax, dt);
  store_act(scale, task, sc, dt);
  for (int c = 0; c < gs; ++c) codes[base + c] = quant_code(load_act(x, base + c, dt), sc, qmax, dt);
}

__global__ void dequantize_kernel(const int8_t* __restrict__ codes, const void* __restrict__ scale,
                                  void* __restrict__ out, int64_t rows, int D, int gs, int dt) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * D) return;
  const int64_t r = i / D;
  const int c = static_cast<int>(i % D);
  const float sc = load_act(scale, r * (D / gs) + c / gs, dt);
  store_act(out, i, dequant(codes[i], sc, dt), dt);
}

__global__ void pack_kernel(const int8_t* __restrict__ codes, uint8_t* __restrict__ packed, int64_t rows, int D,
                            int bits) {
  const int R = row_bytes(D, bits);
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * R) return;
  const int64_t r = i / R;
  packed[i] = pack_byte(codes + r * D, static_cast<int>(i % R), bits);
}

__global__ void unpack_kernel(const uint8_t* __restrict__ packed, int8_t* __restrict__ codes, int64_t rows, int D,
                              int bits) {
  const int R = row_bytes(D, bits);
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * D) return;
  const int64_t r = i / D;
  codes[i] = static_cast<int8_t>(unpack_code(packed + r * R, static_cast<int>(i % D), bits));
}

// one warp per block of `numel` values
__global__ void pack4_kernel(const float* __restrict__ x, uint8_t* __restrict__ packed, uint16_t* __restrict__ sc,
                             int64_t n, int numel) {
  const int64_t blk = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (blk >= n) return;
  const float* src = x + blk * numel;
  float mx = 0.f;
  for (int i = lane; i < numel; i += 32) mx = fmaxf(mx, fabsf(src[i]));
  mx = warp_max(mx);
  const float s = __fdiv_rn(fmaxf(mx, 1e-8f), 7.0f);
  for (int j = lane; j < numel / 2; j += 32) {
    const int lo = nibble_code(src[2 * j], s), hi = nibble_code(src[2 * j + 1], s);
    packed[blk * (numel / 2) + j] = static_cast<uint8_t>((lo & 15) | ((hi & 15) << 4));
  }
  if (lane == 0) sc[blk] = f32_to_f16_bits(s);
}

__global__ void unpack4_kernel(const uint8_t* __restrict__ packed, const uint16_t* __restrict__ sc,
                               float* __restrict__ out, int64_t n, int numel) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n * numel) return;
  const int64_t blk = i / numel;
  out[i] = unpack_nibble(packed + blk * (numel / 2), static_cast<int>(i % numel), f16_bits_to_f32(sc[blk]));
}

static inline unsigned grid_of(int64_t n, int bs) { return static_cast<unsigned>((n + bs - 1) / bs); }

cudaError_t launch_quantize(const void* x, int8_t* codes, void* scale, int64_t rows, int D, int bits, int gs, int dt,
                            cudaStream_t st) {
  const int64_t n = rows * (D / gs);
  if (n == 0) return cudaSuccess;
  quantize_kernel<<<grid_of(n, 256), 256, 0, st>>>(x, codes, scale, rows, D, bits, gs, dt);
  return cudaGetLastError();
}
cudaError_t launch_dequantize(const int8_t* codes, const void* scale, void* out, int64_t rows, int D, int gs, int dt,
                              cudaStream_t st) {
  if (rows * D == 0) return cudaSuccess;
  dequantize_kernel<<<grid_of(rows * D, 256), 256, 0, st>>>(codes, scale, out, rows, D, gs, dt);
  return cudaGetLastError();
}
cudaError_t launch_pack(const int8_t* codes, uint8_t* packed, int64_t rows, int D, int bits, cudaStream_t st) {
  const int64_t n = rows * row_bytes(D, bits);
  if (n == 0) return cudaSuccess;
  pack_kernel<<<grid_of(n, 256), 256, 0, st>>>(codes, packed, rows, D, bits);
  return cudaGetLastError();
}
cudaError_t launch_unpack(const uint8_t* packed, int8_t* codes, int64_t rows, int D, int bits, cudaStream_t st) {
  if (rows * D == 0) return cudaSuccess;
  unpack_kernel<<<grid_of(rows * D, 256), 256, 0, st>>>(packed, codes, rows, D, bits);
  return cudaGetLastError();
}
cudaError_t launch_pack4(const float* x, uint8_t* packed, uint16_t* sc, int64_t n, int numel, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  pack4_kernel<<<grid_of(n, 8), 256, 0, st>>>(x, packed, sc, n, numel);
  return cudaGetLastError();
}
cudaError_t launch_unpack4(const uint8_t* packed, const uint16_t* sc, float* out, int64_t n, int numel,
                           cudaStream_t st) {
  if (n * numel == 0) return cudaSuccess;
  unpack4_kernel<<<grid_of(n * numel, 256), 256, 0, st>>>(packed, sc, out, n, numel);
  return cudaGetLastError();
}

}  // namespace carekv
