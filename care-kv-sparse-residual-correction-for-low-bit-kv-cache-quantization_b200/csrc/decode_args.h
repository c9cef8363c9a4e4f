// Arguments shared by the decode kernels (decode.cu, decode_fast.cu).
#pragma once
#include "common.cuh"

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
  int act_heads;    // query heads per row of q / out (the model's, for a kv-head shard)
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
  int* sel_out;     // [bh][qn][sel_stride]: count, then the selected grid indices
  int sel_stride;   // 1 + p_used * (SK + SV): room for every slot of the grid
  float* kw;        // [bh][qn][p_used*SK][16]: q . R_K per stored K slot and token, written by
                    // the narrow split-K pass when live K scoring runs there; null otherwise
  int s_perm;       // 1: S and kw hold a page's 16 tokens in tok_pos() order
  // fp16 magic keys of the exact low-bit dequantization (3-bit fields at
  // mantissa bit 0, 3, 6 of both halves; 4-bit fields at bit 0, 4; 3-bit
  // field pairs at bits (1, 0), (4, 3), (7, 6), (2, 2), (1, 1), (4, 4),
  // (7, 7), (5, 5) of the low / high half), passed as arguments so the
  // kernels hold them in registers instead of re-creating them per use
  uint32_t dq_keys[13];
  const float* sketch_proj;
  carekv_route_params_t rp;
  int force_generic;  // 1: use the generic split-K pass (tests)
  // prefill correction (route kernel only): every grid row reads cache
  // sequence seq_fixed (>= 0), the attention weights come from attn (laid
  // out like S) instead of exp(S - M) / L, and optional base V rows / page
  // norms replace the cache's dequantised V (the prefill's V_hat with
  // activation-dtype scales)
  int seq_fixed;       // -1: sequence seq_begin + row / H
  const float* attn;   // [bh][qn][p_used*16] attention weights, or null
  const float* o_exact;  // [bh][qn][D] sum_t A V for the exact form (prefill), or null
  const float* v_rows;   // [H][p_used*16][D] or null
  const float* v_pnorm;  // [H][p_used] Frobenius norm of each page's rows, or null
};

// Position of token t (0..15) inside a page's 16 logits: the narrow pass
// stores tokens t and t+8 (t < 8) side by side, at 2t and 2t+1.
__device__ __forceinline__ int tok_pos(int t, int perm) { return perm ? 2 * (t & 7) + (t >> 3) : t; }
// Token held at position j (inverse of tok_pos).
__device__ __forceinline__ int pos_tok(int j, int perm) { return perm ? (j >> 1) + 8 * (j & 1) : j; }

template <int QN>
cudaError_t launch_route(DecodeArgs& a, cudaStream_t st, int n_bh);

template <int QN, int D>
cudaError_t launch_decode_partial_int3(DecodeArgs& a, cudaStream_t st, int n_bh);

template <int QN, int D>
cudaError_t launch_decode_narrow(DecodeArgs& a, cudaStream_t st, int n_bh);
size_t narrow_smem_bytes(const carekv_config_t& c, bool kslot);

}  // namespace carekv
