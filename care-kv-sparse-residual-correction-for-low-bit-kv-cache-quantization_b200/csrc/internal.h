// Host-side launch functions shared between the translation units.
#pragma once
#include <cuda_runtime.h>
#include "../../include/carekv_b200.h"

namespace carekv {
cudaError_t launch_quantize(const void* x, int8_t* codes, void* scale, int64_t rows, int D, int bits, int gs, int dt,
                            cudaStream_t st);
cudaError_t launch_dequantize(const int8_t* codes, const void* scale, void* out, int64_t rows, int D, int gs, int dt,
                              cudaStream_t st);
cudaError_t launch_pack(const int8_t* codes, uint8_t* packed, int64_t rows, int D, int bits, cudaStream_t st);
cudaError_t launch_unpack(const uint8_t* packed, int8_t* codes, int64_t rows, int D, int bits, cudaStream_t st);
cudaError_t launch_pack4(const float* x, uint8_t* packed, uint16_t* sc, int64_t n, int numel, cudaStream_t st);
cudaError_t launch_unpack4(const uint8_t* packed, const uint16_t* sc, float* out, int64_t n, int numel,
                           cudaStream_t st);
// in_H: kv heads per activation row of K / V (the model's, for a kv-head
// shard; the pointers then start at the shard's first head)
cudaError_t launch_prefill_store(const carekv_config_t& cfg, const carekv_cache_t& cache, int layer, const void* K,
                                 const void* V, int T, int seq_begin, int seq_count,
                                 const carekv_store_params_t& prm, const float* sketch_proj, int in_H,
                                 cudaStream_t st);
// the warp-per-page prefill store (store_warp.cu) and the configurations
// and inputs it takes (else launch_prefill_store runs page_store_kernel)
bool prefill_store_warp_supported(const carekv_config_t& cfg, const carekv_cache_t& cache, const void* K,
                                  const void* V, const carekv_store_params_t& prm);
cudaError_t launch_prefill_store_warp(const carekv_config_t& cfg, const carekv_cache_t& cache, int layer,
                                      const void* K, const void* V, int T, int seq_begin, int seq_count,
                                      const carekv_store_params_t& prm, int in_H, cudaStream_t st);
cudaError_t launch_append(const carekv_config_t& cfg, const carekv_cache_t& cache, int layer, const void* k,
                          const void* v, int seq_begin, int seq_count, const carekv_store_params_t& prm,
                          const float* sketch_proj, int may_fill, int in_H, cudaStream_t st);
cudaError_t launch_kivi_k(const void* x, void* out, int64_t n, int T, int D, int bits, int dt, cudaStream_t st);
cudaError_t launch_kivi_v(const void* x, void* out, int64_t rows, int D, int bits, int dt, cudaStream_t st);
struct DecodeArgs;
template <int QN>
cudaError_t launch_decode_generic(DecodeArgs& a, cudaStream_t st, int n_bh);
int decode_attention(const carekv_config_t& cfg, const carekv_cache_t& cache, int layer, const void* q,
                     void* out, int dtype, int seq_begin, int seq_count, int p_used,
                     const carekv_route_params_t& rp, void* ws, size_t ws_bytes, const float* sketch_proj,
                     int act_heads, cudaStream_t st);
size_t workspace_bytes(const carekv_config_t& c, int seq_count, int p_used);
void prepare_decode_streams();               // creates the chunk streams of the current device (not under capture)
int decode_attention_chunks(int seq_count);   // batch chunks one decode attention call runs
size_t prefill_workspace_bytes(const carekv_config_t& c, int n_pos, int p_used);
int prefill_correction(const carekv_config_t& cfg, const carekv_cache_t& cache, int layer, int seq, int n_pos,
                       int p_used, const void* q, const float* logits, const float* row_max, const float* A,
                       const float* A_sum, const float* O, const float* O_exact, const float* v_rows,
                       const float* v_pnorm, void* out, int dtype, const carekv_route_params_t& rp,
                       const float* sketch_proj, void* ws, size_t ws_bytes, cudaStream_t st);
}  // namespace carekv
