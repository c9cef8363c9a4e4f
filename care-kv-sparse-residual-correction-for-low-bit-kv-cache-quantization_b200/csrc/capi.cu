// extern "C" entry points of libcarekv_b200.so: argument validation, buffer
// layout and launch.  See include/carekv_b200.h for the contract of each.
#include <cmath>
#include <cstring>

#include "common.cuh"
#include "internal.h"

using namespace carekv;

namespace {

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

int validate_config(const carekv_config_t* c) {
  if (c == nullptr) return CAREKV_ERR_INVALID_ARG;
  if (c->num_layers < 1 || c->num_kv_heads < 1 || c->num_heads < 1) return CAREKV_ERR_INVALID_ARG;
  if (c->num_heads % c->num_kv_heads != 0) return CAREKV_ERR_INVALID_ARG;
  const int qn = c->num_heads / c->num_kv_heads;
  if (qn != 1 && qn != 2 && qn != 4 && qn != 8) return CAREKV_ERR_UNSUPPORTED;
  if (c->head_dim != 64 && c->head_dim != 128) return CAREKV_ERR_UNSUPPORTED;
  if (c->page_size != kPage) return CAREKV_ERR_UNSUPPORTED;
  if (c->max_pages < 8 || c->max_pages % 8 != 0) return CAREKV_ERR_INVALID_ARG;
  if (c->base_bits < 2 || c->base_bits > 4) return CAREKV_ERR_INVALID_ARG;
  if (c->group_size <= 0 || c->head_dim % c->group_size != 0 || c->group_size % 8 != 0) return CAREKV_ERR_INVALID_ARG;
  if (c->head_dim / c->group_size > 4) return CAREKV_ERR_UNSUPPORTED;
  if (c->k_channel_group != 32) return CAREKV_ERR_UNSUPPORTED;
  if (c->v_token_block <= 0 || kPage % c->v_token_block != 0) return CAREKV_ERR_INVALID_ARG;
  const int C = c->head_dim / c->k_channel_group, NV = kPage / c->v_token_block;
  if (C + NV > 8 || c->v_token_block * c->head_dim / 2 > 256) return CAREKV_ERR_UNSUPPORTED;
  if (c->residual_bits != 4) return CAREKV_ERR_UNSUPPORTED;
  if (c->sketch_dim < 0 || c->sketch_dim > 64) return CAREKV_ERR_INVALID_ARG;
  if (c->scale_mode < CAREKV_SCALE_INT8 || c->scale_mode > CAREKV_SCALE_F32) return CAREKV_ERR_INVALID_ARG;
  if (c->k_slots_per_page < 0 || c->k_slots_per_page > C) return CAREKV_ERR_INVALID_ARG;
  if (c->v_slots_per_page < 0 || c->v_slots_per_page > NV) return CAREKV_ERR_INVALID_ARG;
  if (c->base_kind != CAREKV_BASE_UNIFORM && c->base_kind != CAREKV_BASE_KIVI) return CAREKV_ERR_INVALID_ARG;
  if (c->base_kind == CAREKV_BASE_KIVI) {
    // one V scale per token, scales kept as their activation-dtype values
    if (c->group_size != c->head_dim || c->scale_mode != CAREKV_SCALE_F32) return CAREKV_ERR_INVALID_ARG;
    if (c->kivi_window_pages < 0 || c->kivi_window_pages > c->max_pages) return CAREKV_ERR_INVALID_ARG;
  } else if (c->kivi_window_pages != 0) {
    return CAREKV_ERR_INVALID_ARG;
  }
  return CAREKV_OK;
}

int validate_cache(const carekv_config_t* c, const carekv_cache_t* k) {
  if (k == nullptr || k->batch < 1) return CAREKV_ERR_INVALID_ARG;
  if (!k->k_codes || !k->v_codes || !k->k_scale || !k->v_scale || !k->valid || !k->num_pages || !k->v_norm2 ||
      !k->k_err || !k->v_err || !k->slot_counter || !k->error_flag)
    return CAREKV_ERR_INVALID_ARG;
  if (c->scale_mode == CAREKV_SCALE_INT8 && (!k->k_master || !k->v_master)) return CAREKV_ERR_INVALID_ARG;
  if (c->k_slots_per_page > 0 && (!k->k_slot_group || !k->k_slot_data || !k->k_slot_scale || !k->k_slot_id))
    return CAREKV_ERR_INVALID_ARG;
  if (c->v_slots_per_page > 0 && (!k->v_slot_block || !k->v_slot_data || !k->v_slot_scale || !k->v_slot_id))
    return CAREKV_ERR_INVALID_ARG;
  if (c->base_kind == CAREKV_BASE_KIVI && (!k->k_chan_scale || !k->prefill_tokens ||
                                           (c->kivi_window_pages > 0 && !k->k_window)))
    return CAREKV_ERR_INVALID_ARG;
  // the kernels stage rows, scales and slot payloads with 16-byte and bulk
  // copies: every buffer starts on a 16-byte boundary (cudaMalloc gives 256)
  const void* bufs[] = {k->k_codes, k->v_codes, k->k_scale, k->v_scale, k->k_master, k->v_master, k->valid,
                        k->num_pages, k->v_norm2, k->k_slot_group, k->k_slot_data, k->k_slot_scale, k->k_slot_id,
                        k->v_slot_block, k->v_slot_data, k->v_slot_scale, k->v_slot_id, k->k_err, k->v_err,
                        k->k_sketch, k->slot_counter, k->read_counter, k->error_flag, k->k_chan_scale,
                        k->k_window, k->prefill_tokens};
  for (const void* b : bufs)
    if ((reinterpret_cast<uintptr_t>(b) & 15) != 0) return CAREKV_ERR_INVALID_ARG;
  return CAREKV_OK;
}

int validate_range(const carekv_cache_t* k, int32_t layer, int32_t seq_begin, int32_t seq_count,
                   const carekv_config_t* c) {
  if (layer < 0 || layer >= c->num_layers) return CAREKV_ERR_INVALID_ARG;
  if (seq_begin < 0 || seq_count < 0 || seq_begin + seq_count > k->batch) return CAREKV_ERR_INVALID_ARG;
  return CAREKV_OK;
}

int validate_dtype(int32_t dt) {
  return (dt == CAREKV_F32 || dt == CAREKV_F16 || dt == CAREKV_BF16) ? CAREKV_OK : CAREKV_ERR_INVALID_ARG;
}

int cuda_status(cudaError_t e) { return e == cudaSuccess ? CAREKV_OK : CAREKV_ERR_CUDA; }

// A kv-head shard: the arena's kv heads are [kvh_begin, kvh_begin + H) of a
// model with kvh_total kv heads.
int validate_shard(const carekv_config_t* c, const carekv_shard_t* sh) {
  if (sh == nullptr || sh->kvh_begin < 0 || sh->kvh_total < c->num_kv_heads ||
      sh->kvh_begin + c->num_kv_heads > sh->kvh_total)
    return CAREKV_ERR_INVALID_ARG;
  return CAREKV_OK;
}

int64_t act_bytes(int32_t dt) { return dt == CAREKV_F32 ? 4 : 2; }

// The cached router: sketch K scores, a known policy and score; its
// adaptive_score thresholds work on at most 32 selected slots per query
// (absolute caps).
int validate_legacy(const carekv_route_params_t* p) {
  if (p->legacy == 0) return CAREKV_OK;
  if (p->legacy != 1 || p->kscore_live) return CAREKV_ERR_INVALID_ARG;
  if (p->policy < CAREKV_POLICY_SEPARATE || p->policy > CAREKV_POLICY_ADAPTIVE) return CAREKV_ERR_INVALID_ARG;
  if (p->baseline_score < CAREKV_SCORE_CAREKV || p->baseline_score > CAREKV_SCORE_ORACLE_PROXY)
    return CAREKV_ERR_INVALID_ARG;
  if (p->adaptive_score && (p->budget_mode != 0 || p->read_k + p->read_v > 32)) return CAREKV_ERR_UNSUPPORTED;
  return CAREKV_OK;
}

#define CHECK(x)                      \
  do {                                \
    const int _s = (x);               \
    if (_s != CAREKV_OK) return _s;   \
  } while (0)

}  // namespace

extern "C" {

int carekv_abi_version(void) { return CAREKV_ABI_VERSION; }

const char* carekv_status_string(int status) {
  switch (status) {
    case CAREKV_OK: return "ok";
    case CAREKV_ERR_INVALID_ARG: return "invalid argument";
    case CAREKV_ERR_UNSUPPORTED: return "unsupported configuration";
    case CAREKV_ERR_CACHE_FULL: return "KV cache is full";
    case CAREKV_ERR_CUDA: return "CUDA error";
    case CAREKV_ERR_WORKSPACE: return "workspace too small";
    case CAREKV_ERR_DEVICE_CHECK: return "device-side check failed";
    default: return "unknown status";
  }
}

int carekv_cache_layout(const carekv_config_t* cfg, int32_t batch, size_t sizes[CAREKV_NUM_BUFFERS]) {
  CHECK(validate_config(cfg));
  if (batch < 1 || sizes == nullptr) return CAREKV_ERR_INVALID_ARG;
  const Dims d = make_dims(*cfg);
  const size_t pages = static_cast<size_t>(batch) * d.L * d.H * d.P;
  const size_t rows = pages * kPage;
  size_t i = 0;
  sizes[i++] = rows * d.R;                                   // k_codes
  sizes[i++] = rows * d.R;                                   // v_codes
  sizes[i++] = rows * d.G * d.scale_elem;                    // k_scale
  sizes[i++] = rows * d.G * d.scale_elem;                    // v_scale
  sizes[i++] = cfg->scale_mode == CAREKV_SCALE_INT8 ? pages * 2 : 0;  // k_master
  sizes[i++] = cfg->scale_mode == CAREKV_SCALE_INT8 ? pages * 2 : 0;  // v_master
  sizes[i++] = pages * 4;                                    // valid
  sizes[i++] = static_cast<size_t>(batch) * d.L * d.H * 4;   // num_pages
  sizes[i++] = pages * 4;                                    // v_norm2
  sizes[i++] = pages * d.SK;                                 // k_slot_group
  sizes[i++] = pages * d.SK * d.kslot_bytes;                 // k_slot_data
  sizes[i++] = pages * d.SK * 2;                             // k_slot_scale
  sizes[i++] = pages * d.SK * 4;                             // k_slot_id
  sizes[i++] = pages * d.SV;                                 // v_slot_block
  sizes[i++] = pages * d.SV * d.vslot_bytes;                 // v_slot_data
  sizes[i++] = pages * d.SV * 2;                             // v_slot_scale
  sizes[i++] = pages * d.SV * 4;                             // v_slot_id
  sizes[i++] = pages * d.C * 2;                              // k_err
  sizes[i++] = pages * d.NV * 2;                             // v_err
  sizes[i++] = pages * d.C * d.sketch * 2;                   // k_sketch
  sizes[i++] = static_cast<size_t>(batch) * 2 * 4;           // slot_counter
  sizes[i++] = static_cast<size_t>(d.L) * d.H * 2 * 8;       // read_counter
  sizes[i++] = 4;                                            // error_flag
  const size_t lh = static_cast<size_t>(batch) * d.L * d.H;
  const bool kivi = cfg->base_kind == CAREKV_BASE_KIVI;
  sizes[i++] = kivi ? lh * d.D * 4 : 0;                                          // k_chan_scale
  sizes[i++] = kivi ? lh * static_cast<size_t>(cfg->kivi_window_pages) * kPage * d.D * 2 : 0;  // k_window
  sizes[i++] = kivi ? lh * 4 : 0;                                                // prefill_tokens
  return CAREKV_OK;
}

int carekv_cache_init(const carekv_config_t* cfg, const carekv_cache_t* cache, void* stream) {
  CHECK(validate_config(cfg));
  CHECK(validate_cache(cfg, cache));
  size_t sz[CAREKV_NUM_BUFFERS];
  CHECK(carekv_cache_layout(cfg, cache->batch, sz));
  void* ptrs[CAREKV_NUM_BUFFERS] = {
      cache->k_codes,      cache->v_codes,      cache->k_scale,      cache->v_scale,     cache->k_master,
      cache->v_master,     cache->valid,        cache->num_pages,    cache->v_norm2,     cache->k_slot_group,
      cache->k_slot_data,  cache->k_slot_scale, cache->k_slot_id,    cache->v_slot_block, cache->v_slot_data,
      cache->v_slot_scale, cache->v_slot_id,    cache->k_err,        cache->v_err,       cache->k_sketch,
      cache->slot_counter, cache->read_counter, cache->error_flag, cache->k_chan_scale,
      cache->k_window,     cache->prefill_tokens};
  // slot tables start empty (-1); everything else starts at zero
  const bool minus_one[CAREKV_NUM_BUFFERS] = {false, false, false, false, false, false, false, false,
                                              false, true,  false, false, true,  true,  false, false,
                                              true,  false, false, false, false, false, false, false,
                                              false, false};
  prepare_decode_streams();
  cudaStream_t st = as_stream(stream);
  for (int i = 0; i < CAREKV_NUM_BUFFERS; ++i) {
    if (ptrs[i] == nullptr || sz[i] == 0) continue;
    CHECK(cuda_status(cudaMemsetAsync(ptrs[i], minus_one[i] ? 0xFF : 0, sz[i], st)));
  }
  return CAREKV_OK;
}

int carekv_quantize(const void* x, int8_t* codes, void* scale, int64_t rows, int32_t D, int32_t bits,
                    int32_t group_size, int32_t dtype, void* stream) {
  if (!x || !codes || !scale || rows < 0 || D <= 0 || group_size <= 0 || D % group_size) return CAREKV_ERR_INVALID_ARG;
  if (bits < 2 || bits > 4) return CAREKV_ERR_INVALID_ARG;
  CHECK(validate_dtype(dtype));
  return cuda_status(launch_quantize(x, codes, scale, rows, D, bits, group_size, dtype, as_stream(stream)));
}

int carekv_kivi_quant_dequant_k(const void* K, void* out, int64_t n, int32_t T, int32_t D, int32_t bits,
                                int32_t dtype, void* stream) {
  if (!K || !out || n < 0 || T < 0 || D <= 0 || bits < 2 || bits > 8) return CAREKV_ERR_INVALID_ARG;
  CHECK(validate_dtype(dtype));
  return cuda_status(launch_kivi_k(K, out, n, T, D, bits, dtype, as_stream(stream)));
}

int carekv_kivi_quant_dequant_v(const void* V, void* out, int64_t rows, int32_t D, int32_t bits, int32_t dtype,
                                void* stream) {
  if (!V || !out || rows < 0 || D <= 0 || bits < 2 || bits > 8) return CAREKV_ERR_INVALID_ARG;
  CHECK(validate_dtype(dtype));
  return cuda_status(launch_kivi_v(V, out, rows, D, bits, dtype, as_stream(stream)));
}

int carekv_dequantize(const int8_t* codes, const void* scale, void* out, int64_t rows, int32_t D,
                      int32_t group_size, int32_t dtype, void* stream) {
  if (!codes || !scale || !out || rows < 0 || D <= 0 || group_size <= 0 || D % group_size) return CAREKV_ERR_INVALID_ARG;
  CHECK(validate_dtype(dtype));
  return cuda_status(launch_dequantize(codes, scale, out, rows, D, group_size, dtype, as_stream(stream)));
}

int carekv_pack_codes(const int8_t* codes, uint8_t* packed, int64_t rows, int32_t D, int32_t bits, void* stream) {
  if (!codes || !packed || rows < 0 || bits < 2 || bits > 4) return CAREKV_ERR_INVALID_ARG;
  if (D <= 0 || (bits == 3 && D % 8) || (bits == 2 && D % 4) || (bits == 4 && D % 2)) return CAREKV_ERR_INVALID_ARG;
  return cuda_status(launch_pack(codes, packed, rows, D, bits, as_stream(stream)));
}

int carekv_unpack_codes(const uint8_t* packed, int8_t* codes, int64_t rows, int32_t D, int32_t bits, void* stream) {
  if (!codes || !packed || rows < 0 || bits < 2 || bits > 4) return CAREKV_ERR_INVALID_ARG;
  if (D <= 0 || (bits == 3 && D % 8) || (bits == 2 && D % 4) || (bits == 4 && D % 2)) return CAREKV_ERR_INVALID_ARG;
  return cuda_status(launch_unpack(packed, codes, rows, D, bits, as_stream(stream)));
}

int carekv_pack_4bit(const float* x, uint8_t* packed, uint16_t* scale_f16, int64_t n, int32_t numel, void* stream) {
  if (!x || !packed || !scale_f16 || n < 0 || numel <= 0 || numel % 2) return CAREKV_ERR_INVALID_ARG;
  return cuda_status(launch_pack4(x, packed, scale_f16, n, numel, as_stream(stream)));
}

int carekv_unpack_4bit(const uint8_t* packed, const uint16_t* scale_f16, float* out, int64_t n, int32_t numel,
                       void* stream) {
  if (!out || !packed || !scale_f16 || n < 0 || numel <= 0 || numel % 2) return CAREKV_ERR_INVALID_ARG;
  return cuda_status(launch_unpack4(packed, scale_f16, out, n, numel, as_stream(stream)));
}

static int validate_store_params(const carekv_config_t* cfg, const carekv_store_params_t* p) {
  if (p == nullptr) return CAREKV_ERR_INVALID_ARG;
  CHECK(validate_dtype(p->input_dtype));
  if (p->decode_page_master != 0 && p->decode_page_master != 1) return CAREKV_ERR_INVALID_ARG;
  const int C = cfg->head_dim / cfg->k_channel_group, NV = kPage / cfg->v_token_block;
  if (p->k_budget < 0 || p->v_budget < 0) return CAREKV_ERR_INVALID_ARG;
  if (p->joint_budget > 0) {
    if (cfg->k_slots_per_page < std::min(p->joint_budget, C) || cfg->v_slots_per_page < std::min(p->joint_budget, NV))
      return CAREKV_ERR_INVALID_ARG;
  } else if (std::min(p->k_budget, C) > cfg->k_slots_per_page || std::min(p->v_budget, NV) > cfg->v_slots_per_page) {
    return CAREKV_ERR_INVALID_ARG;
  }
  return CAREKV_OK;
}

int carekv_prefill_store(const carekv_config_t* cfg, const carekv_cache_t* cache, int32_t layer, const void* K,
                         const void* V, int32_t T, int32_t seq_begin, int32_t seq_count,
                         const carekv_store_params_t* params, const float* sketch_proj, void* stream) {
  CHECK(validate_config(cfg));
  const carekv_shard_t whole = {0, cfg->num_kv_heads};
  return carekv_prefill_store_shard(cfg, cache, layer, K, V, T, seq_begin, seq_count, params, sketch_proj, &whole,
                                    stream);
}

int carekv_prefill_store_shard(const carekv_config_t* cfg, const carekv_cache_t* cache, int32_t layer,
                               const void* K, const void* V, int32_t T, int32_t seq_begin, int32_t seq_count,
                               const carekv_store_params_t* params, const float* sketch_proj,
                               const carekv_shard_t* shard, void* stream) {
  CHECK(validate_config(cfg));
  CHECK(validate_shard(cfg, shard));
  CHECK(validate_cache(cfg, cache));
  CHECK(validate_range(cache, layer, seq_begin, seq_count, cfg));
  CHECK(validate_store_params(cfg, params));
  if (T < 0 || (T > 0 && (!K || !V))) return CAREKV_ERR_INVALID_ARG;
  if ((T + kPage - 1) / kPage > cfg->max_pages) return CAREKV_ERR_CACHE_FULL;
  if (cfg->sketch_dim > 0 && cache->k_sketch && !sketch_proj) return CAREKV_ERR_INVALID_ARG;
  const int64_t off = static_cast<int64_t>(shard->kvh_begin) * T * cfg->head_dim * act_bytes(params->input_dtype);
  return cuda_status(launch_prefill_store(*cfg, *cache, layer, static_cast<const char*>(K) + off,
                                          static_cast<const char*>(V) + off, T, seq_begin, seq_count, *params,
                                          sketch_proj, shard->kvh_total, as_stream(stream)));
}

int carekv_append(const carekv_config_t* cfg, const carekv_cache_t* cache, int32_t layer, const void* k,
                  const void* v, int32_t seq_begin, int32_t seq_count, const carekv_store_params_t* params,
                  const float* sketch_proj, int32_t may_fill_page, void* stream) {
  CHECK(validate_config(cfg));
  const carekv_shard_t whole = {0, cfg->num_kv_heads};
  return carekv_append_shard(cfg, cache, layer, k, v, seq_begin, seq_count, params, sketch_proj, may_fill_page,
                             &whole, stream);
}

int carekv_append_shard(const carekv_config_t* cfg, const carekv_cache_t* cache, int32_t layer, const void* k,
                        const void* v, int32_t seq_begin, int32_t seq_count, const carekv_store_params_t* params,
                        const float* sketch_proj, int32_t may_fill_page, const carekv_shard_t* shard,
                        void* stream) {
  CHECK(validate_config(cfg));
  CHECK(validate_shard(cfg, shard));
  CHECK(validate_cache(cfg, cache));
  CHECK(validate_range(cache, layer, seq_begin, seq_count, cfg));
  CHECK(validate_store_params(cfg, params));
  if (seq_count > 0 && (!k || !v)) return CAREKV_ERR_INVALID_ARG;
  if (cfg->sketch_dim > 0 && cache->k_sketch && !sketch_proj) return CAREKV_ERR_INVALID_ARG;
  const int64_t off = static_cast<int64_t>(shard->kvh_begin) * cfg->head_dim * act_bytes(params->input_dtype);
  return cuda_status(launch_append(*cfg, *cache, layer, static_cast<const char*>(k) + off,
                                   static_cast<const char*>(v) + off, seq_begin, seq_count, *params, sketch_proj,
                                   may_fill_page != 0, shard->kvh_total, as_stream(stream)));
}

int carekv_decode_workspace_bytes(const carekv_config_t* cfg, int32_t seq_count, int32_t max_pages_used,
                                  size_t* bytes) {
  CHECK(validate_config(cfg));
  if (!bytes || seq_count < 0 || max_pages_used < 0 || max_pages_used > cfg->max_pages) return CAREKV_ERR_INVALID_ARG;
  *bytes = workspace_bytes(*cfg, seq_count, max_pages_used);
  return CAREKV_OK;
}

int carekv_decode_attention(const carekv_config_t* cfg, const carekv_cache_t* cache, int32_t layer, const void* q,
                            void* out, int32_t dtype, int32_t seq_begin, int32_t seq_count, int32_t max_pages_used,
                            const carekv_route_params_t* params, const float* sketch_proj, void* workspace,
                            size_t workspace_bytes_, void* stream) {
  CHECK(validate_config(cfg));
  const carekv_shard_t whole = {0, cfg->num_kv_heads};
  return carekv_decode_attention_shard(cfg, cache, layer, q, out, dtype, seq_begin, seq_count, max_pages_used,
                                       params, sketch_proj, workspace, workspace_bytes_, &whole, stream);
}

int carekv_decode_attention_shard(const carekv_config_t* cfg, const carekv_cache_t* cache, int32_t layer,
                                  const void* q, void* out, int32_t dtype, int32_t seq_begin, int32_t seq_count,
                                  int32_t max_pages_used, const carekv_route_params_t* params,
                                  const float* sketch_proj, void* workspace, size_t workspace_bytes_,
                                  const carekv_shard_t* shard, void* stream) {
  CHECK(validate_config(cfg));
  CHECK(validate_shard(cfg, shard));
  CHECK(validate_cache(cfg, cache));
  CHECK(validate_range(cache, layer, seq_begin, seq_count, cfg));
  CHECK(validate_dtype(dtype));
  if (!params || !q || !out || !workspace) return CAREKV_ERR_INVALID_ARG;
  if (max_pages_used < 0 || max_pages_used > cfg->max_pages) return CAREKV_ERR_INVALID_ARG;
  if (params->kind < CAREKV_KIND_BOTH || params->kind > CAREKV_KIND_NONE) return CAREKV_ERR_INVALID_ARG;
  if (params->kind != CAREKV_KIND_NONE) {
    // any budget is served (selections beyond 32 entries apply in rounds)
    if (params->budget_mode == 0 && (params->read_k < 0 || params->read_v < 0)) return CAREKV_ERR_INVALID_ARG;
    if (!params->kscore_live && (!cache->k_sketch || cfg->sketch_dim <= 0 || !sketch_proj))
      return CAREKV_ERR_INVALID_ARG;
    CHECK(validate_legacy(params));
  }
  if (seq_count == 0 || max_pages_used == 0) {
    if (seq_count == 0) return CAREKV_OK;
  }
  const int qn = cfg->num_heads / cfg->num_kv_heads;
  const int64_t off = static_cast<int64_t>(shard->kvh_begin) * qn * cfg->head_dim * act_bytes(dtype);
  return decode_attention(*cfg, *cache, layer, static_cast<const char*>(q) + off, static_cast<char*>(out) + off, dtype,
                          seq_begin, seq_count, std::max(1, max_pages_used), *params, workspace, workspace_bytes_,
                          sketch_proj, shard->kvh_total * qn, as_stream(stream));
}

int carekv_prefill_workspace_bytes(const carekv_config_t* cfg, int32_t n_pos, int32_t max_pages_used,
                                   size_t* bytes) {
  CHECK(validate_config(cfg));
  if (!bytes || n_pos < 0 || max_pages_used < 1 || max_pages_used > cfg->max_pages) return CAREKV_ERR_INVALID_ARG;
  *bytes = prefill_workspace_bytes(*cfg, n_pos, max_pages_used);
  return CAREKV_OK;
}

int carekv_prefill_correction(const carekv_config_t* cfg, const carekv_cache_t* cache, int32_t layer, int32_t seq,
                              int32_t n_pos, int32_t max_pages_used, const void* q, const float* logits,
                              const float* row_max, const float* attn, const float* attn_sum,
                              const float* o_base, const float* o_exact, const float* v_rows,
                              const float* v_pnorm, void* out,
                              int32_t dtype, const carekv_route_params_t* params, const float* sketch_proj,
                              void* workspace,
                              size_t workspace_bytes_, void* stream) {
  CHECK(validate_config(cfg));
  CHECK(validate_cache(cfg, cache));
  CHECK(validate_range(cache, layer, seq, 1, cfg));
  CHECK(validate_dtype(dtype));
  if (!params || !q || !attn || !o_base || !out || !workspace) return CAREKV_ERR_INVALID_ARG;
  if (n_pos < 0 || max_pages_used < 1 || max_pages_used > cfg->max_pages) return CAREKV_ERR_INVALID_ARG;
  if (params->kind < CAREKV_KIND_BOTH || params->kind > CAREKV_KIND_NONE) return CAREKV_ERR_INVALID_ARG;
  // the sketch proxy reads the logits and their row maxima (and the sketches)
  if (params->kind != CAREKV_KIND_NONE && !params->kscore_live &&
      (!logits || !row_max || !cache->k_sketch || cfg->sketch_dim <= 0 || !sketch_proj))
    return CAREKV_ERR_INVALID_ARG;
  if (params->kind != CAREKV_KIND_NONE) {
    // any budget is served (selections beyond 32 entries apply in rounds)
    if (params->budget_mode == 0 && (params->read_k < 0 || params->read_v < 0)) return CAREKV_ERR_INVALID_ARG;
    CHECK(validate_legacy(params));
  }
  if (n_pos == 0) return CAREKV_OK;
  return prefill_correction(*cfg, *cache, layer, seq, n_pos, max_pages_used, q, logits, row_max, attn, attn_sum,
                            o_base, o_exact, v_rows, v_pnorm, out, dtype, *params, sketch_proj, workspace,
                            workspace_bytes_, as_stream(stream));
}

int carekv_decode_attention_launches(const carekv_config_t* cfg, int32_t seq_count, int32_t* launches) {
  CHECK(validate_config(cfg));
  if (!launches || seq_count < 0) return CAREKV_ERR_INVALID_ARG;
  *launches = 2 * decode_attention_chunks(seq_count);
  return CAREKV_OK;
}

int carekv_check_device_errors(const carekv_cache_t* cache, int32_t* flags_out, void* stream) {
  if (!cache || !cache->error_flag) return CAREKV_ERR_INVALID_ARG;
  int32_t h = 0;
  cudaStream_t st = as_stream(stream);
  CHECK(cuda_status(cudaMemcpyAsync(&h, cache->error_flag, sizeof(int32_t), cudaMemcpyDeviceToHost, st)));
  CHECK(cuda_status(cudaStreamSynchronize(st)));
  if (h != 0) CHECK(cuda_status(cudaMemsetAsync(cache->error_flag, 0, sizeof(int32_t), st)));
  if (flags_out) *flags_out = h;
  if (h & kErrPageOverflow) return CAREKV_ERR_CACHE_FULL;
  return h ? CAREKV_ERR_DEVICE_CHECK : CAREKV_OK;
}

}  // extern "C"
