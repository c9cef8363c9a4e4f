/*
 * carekv_b200.h -- C ABI of the B200 CARE-KV decode hot path.
 *
 * Plain C: pointers, sizes and status codes; no framework types.  Every
 * device pointer is caller-owned device memory; every entry point takes an
 * explicit CUDA stream (cudaStream_t passed as void*) and returns
 * CAREKV_OK or an error code.  Nothing here allocates device memory except
 * where a comment says otherwise.
 *
 * Reference interfaces replaced (paths relative to the reference project):
 *   quantizer.py:31-99, 257-383     -> carekv_quantize / carekv_dequantize /
 *                                      carekv_pack_codes / carekv_unpack_codes
 *   residual_store.py:121-146       -> carekv_pack_4bit / carekv_unpack_4bit
 *   kivi_helpers.py:35-59           -> carekv_kivi_quant_dequant_k / _v
 *   cache.py:430-536 (buffers)      -> carekv_cache_layout / carekv_cache_init
 *   layer.py:204-334 + cache.py:617-654 + residual_store.py:239-464
 *                                   -> carekv_prefill_store
 *   layer.py:1028-1146 + cache.py:656-701
 *                                   -> carekv_append
 *   attention.py:979-1039 (base decode) + attention.py:576-957
 *   (vectorized_joint_correction) + residual_router.py:37-76
 *                                   -> carekv_decode_attention
 *   layer.py:458-637 (_apply_sparse_prefill_correction_stored, vectorized
 *   router) + attention.py:576-957  -> carekv_prefill_correction
 */
#ifndef CAREKV_B200_H
#define CAREKV_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CAREKV_ABI_VERSION 2

/* status codes */
#define CAREKV_OK                 0
#define CAREKV_ERR_INVALID_ARG    1   /* bad pointer, size or config value      */
#define CAREKV_ERR_UNSUPPORTED    2   /* valid but not built (e.g. page_size!=16) */
#define CAREKV_ERR_CACHE_FULL     3   /* a page beyond max_pages was needed      */
#define CAREKV_ERR_CUDA           4   /* a CUDA launch or API call failed        */
#define CAREKV_ERR_WORKSPACE      5   /* workspace smaller than required         */
#define CAREKV_ERR_DEVICE_CHECK   6   /* a device-side bounds check tripped      */

/* activation element types */
#define CAREKV_F32   0
#define CAREKV_F16   1
#define CAREKV_BF16  2

/* base scale storage (CacheConfig.scale_quant / scale_dtype) */
#define CAREKV_SCALE_INT8  0   /* int8 codes + one fp16 master per page */
#define CAREKV_SCALE_F16   1
#define CAREKV_SCALE_BF16  2
#define CAREKV_SCALE_F32   3

/* base quantizer of an arena (CacheConfig.base_quantizer) */
#define CAREKV_BASE_UNIFORM 0   /* per-group INT-b codes and scales ("uniform")          */
#define CAREKV_BASE_KIVI    1   /* KIVI style ("kivi_style" / "kvquant_style"): prefill K
                                 * codes with one scale per channel over the prefill,
                                 * V codes with one scale per token; decode-appended K
                                 * rows kept in fp16 (kivi_helpers.py:35-59,
                                 * layer.py:1037-1085)                                  */

/* Static shape of one cache arena (CacheConfig, cache.py:209-384). */
typedef struct carekv_config {
    int32_t num_layers;
    int32_t num_heads;          /* query heads                                */
    int32_t num_kv_heads;
    int32_t head_dim;           /* 64 or 128                                  */
    int32_t page_size;          /* tokens per page; 16                        */
    int32_t max_pages;          /* per (sequence, layer, kv head), multiple of 8 */
    int32_t base_bits;          /* 2, 3 or 4                                  */
    int32_t group_size;         /* per-group quantization width; divides head_dim */
    int32_t k_channel_group;    /* channels per K residual slot; 32           */
    int32_t v_token_block;      /* tokens per V residual slot; divides page_size */
    int32_t sketch_dim;         /* fp16 sketch length per K group, 0 = none kept */
    int32_t residual_bits;      /* 4                                          */
    int32_t scale_mode;         /* CAREKV_SCALE_*                             */
    int32_t k_slots_per_page;   /* K slot capacity per page (>= store budget)  */
    int32_t v_slots_per_page;   /* V slot capacity per page                    */
    int32_t base_kind;          /* CAREKV_BASE_*; KIVI needs group_size == head_dim
                                 * (one V scale per token) and scale_mode F32 (the
                                 * scales' activation-dtype values)             */
    int32_t kivi_window_pages;  /* KIVI: pages of fp16 K rows per (sequence, layer,
                                 * kv head) for decode-appended tokens; 0 otherwise */
} carekv_config_t;

/* Device buffers of one arena holding `batch` sequences.  Shapes use
 * B=batch, L=num_layers, H=num_kv_heads, P=max_pages, T=page_size,
 * R=packed row bytes, G=head_dim/group_size, C=head_dim/k_channel_group,
 * NV=page_size/v_token_block, SK/SV=slot capacities.  Every buffer starts on
 * a 16-byte boundary (cudaMalloc gives 256); a misaligned one is rejected
 * with CAREKV_ERR_INVALID_ARG. */
typedef struct carekv_cache {
    int32_t   batch;
    uint8_t  *k_codes;        /* [B][L][H][P][T][R] packed rows (quantizer.py row format) */
    uint8_t  *v_codes;
    void     *k_scale;        /* [B][L][H][P][T][G] int8 | fp16 | bf16 | fp32              */
    void     *v_scale;
    uint16_t *k_master;       /* [B][L][H][P] fp16 bits; int8 scale mode only              */
    uint16_t *v_master;
    int32_t  *valid;          /* [B][L][H][P] valid rows per page                          */
    int32_t  *num_pages;      /* [B][L][H] allocated pages                                 */
    float    *v_norm2;        /* [B][L][H][P] sum of squared dequantized V over valid rows */
    int8_t   *k_slot_group;   /* [B][L][H][P][SK] channel group of each kept K slot, ascending, -1 = empty */
    uint8_t  *k_slot_data;    /* [B][L][H][P][SK][T*k_channel_group/2] 4-bit payload        */
    uint16_t *k_slot_scale;   /* [B][L][H][P][SK] fp16 bits                                 */
    int32_t  *k_slot_id;      /* [B][L][H][P][SK] id the reference arena would assign       */
    int8_t   *v_slot_block;   /* [B][L][H][P][SV] token block of each kept V slot           */
    uint8_t  *v_slot_data;    /* [B][L][H][P][SV][v_token_block*head_dim/2]                 */
    uint16_t *v_slot_scale;   /* [B][L][H][P][SV]                                           */
    int32_t  *v_slot_id;      /* [B][L][H][P][SV]                                           */
    uint16_t *k_err;          /* [B][L][H][P][C] fp16 mean residual row norm per K group    */
    uint16_t *v_err;          /* [B][L][H][P][NV]                                           */
    uint16_t *k_sketch;       /* [B][L][H][P][C][sketch_dim] fp16, may be NULL              */
    int32_t  *slot_counter;   /* [B][2] next K / V arena id per sequence                    */
    unsigned long long *read_counter; /* [L][H][2] K / V slots read, may be NULL           */
    int32_t  *error_flag;     /* [1] bit mask set by device-side checks                    */
    /* KIVI base only (NULL otherwise): */
    float    *k_chan_scale;   /* [B][L][H][D] per-channel K scale of the prefill (dtype value) */
    uint16_t *k_window;       /* [B][L][H][W][T][D] fp16 K rows appended by decode: page
                               * prefill_tokens / T + w of the sequence is window page w   */
    int32_t  *prefill_tokens; /* [B][L][H] tokens written by the (single) prefill          */
} carekv_cache_t;

/* Per-call store policy, resolved by the host for one layer
 * (residual_store.py:370-423, cache.py:180-202). */
typedef struct carekv_store_params {
    int32_t k_budget;         /* K slots kept per page (<= k_slots_per_page)   */
    int32_t v_budget;
    int32_t joint_budget;     /* > 0 selects the legacy joint policy          */
    int32_t store_nothing;    /* 1: keep no slot (ratio 0 everywhere)         */
    int32_t sink_tokens;      /* rows with absolute position < this are sink  */
    int32_t token_start;      /* absolute position of the first prefill row   */
    float   sensitivity;      /* layer sensitivity                            */
    int32_t input_dtype;      /* CAREKV_F32 / F16 / BF16 of the K and V rows   */
    int32_t decode_page_master; /* int8 scales: 0 = a page opened by decode keeps
                                 * master 0, so its rows read back as 0 (the
                                 * reference, cache.py:689-695); 1 = its first
                                 * appended row sets the master (max scale / 127,
                                 * as write_base does, cache.py:592-606); later
                                 * rows keep it, so a later group scale above
                                 * 127 x master saturates at int8 code 127 and
                                 * that row reads back clipped (write_base takes
                                 * the largest scale of the whole page)         */
} carekv_store_params_t;

/* Per-call routing / correction policy (attention.py:576-957,
 * residual_router.py:37-76), resolved by the host for one layer. */
#define CAREKV_KIND_BOTH 0
#define CAREKV_KIND_K    1
#define CAREKV_KIND_V    2
#define CAREKV_KIND_NONE 3    /* base attention only */
typedef struct carekv_route_params {
    int32_t kind;             /* CAREKV_KIND_*                                */
    int32_t joint;            /* 1 joint top-k over K and V, 0 separate       */
    int32_t score_normalize;  /* per-query mean normalisation                  */
    int32_t kscore_live;      /* 1 combined_kvscore, 0 sketch proxy score      */
    int32_t exact;            /* 1 exact softmax K correction, 0 linear        */
    int32_t budget_mode;      /* 0 absolute (read_k/read_v), 1 ratio           */
    int32_t read_k;
    int32_t read_v;
    double  ratio_k;          /* ratio mode; double so int(n * ratio) matches Python */
    double  ratio_v;
    float   k_corr_scale;     /* linear mode only                              */
    float   sensitivity;
    float   lambda_k;
    float   lambda_v;
    /* The cached router (correction_impl "python" / "cached"): when legacy is
     * 1 the selection follows ResidualRouter.route (residual_router.py:88-452)
     * and the correction apply_slot_corrections (attention.py:208-374): K
     * slots scored from their sketches (kscore_live must be 0), score
     * normalisation whenever kind is "both", the policies below, and the
     * adaptive_score thresholds on the selected slots.  0: the vectorized
     * router (attention.py:576-957). */
    int32_t legacy;
    int32_t policy;           /* legacy: CAREKV_POLICY_*                            */
    int32_t baseline_score;   /* legacy: CAREKV_SCORE_* (baseline_score ablations)  */
    int32_t adaptive_score;   /* legacy: 1 = read_budget_mode "adaptive_score"      */
    float   rel_threshold;    /* read_relative_threshold                            */
    float   abs_threshold;    /* read_absolute_threshold                            */
    int32_t min_keep;         /* read_min_keep                                      */
} carekv_route_params_t;
#define CAREKV_POLICY_SEPARATE 0
#define CAREKV_POLICY_JOINT    1
#define CAREKV_POLICY_K_FIRST  2
#define CAREKV_POLICY_ADAPTIVE 3
#define CAREKV_SCORE_CAREKV         0   /* mass x |q.k sketch| x boundary x V diff x sens */
#define CAREKV_SCORE_MAGNITUDE_ONLY 1
#define CAREKV_SCORE_ATTENTION_ONLY 2
#define CAREKV_SCORE_ORACLE_PROXY   3

/* ABI version and a static string for a status code. */
int carekv_abi_version(void);
const char *carekv_status_string(int status);

/* Byte sizes of the arena buffers, in the order of carekv_cache_t's pointer
 * fields (26 entries, k_codes .. prefill_tokens; the last three are 0 for a
 * uniform base).  Replaces the sizing in cache.py:430-536 (the KIVI fp16
 * side buffer, cache.py:487-499, becomes packed codes, scales and a bounded
 * fp16 window). */
#define CAREKV_NUM_BUFFERS 26
int carekv_cache_layout(const carekv_config_t *cfg, int32_t batch, size_t sizes[CAREKV_NUM_BUFFERS]);

/* Reset an arena to empty: counters, valid rows and page counts zeroed,
 * slot tables set to -1.  Replaces CAREKVCache._init_buffers (cache.py:430-536). */
int carekv_cache_init(const carekv_config_t *cfg, const carekv_cache_t *cache, void *stream);

/* ---- standalone quantizer ops on contiguous device rows ------------------ */
/* quantize (quantizer.py:31-64): x [rows][D] -> codes int8 [rows][D],
 * scale [rows][D/g] in the same dtype as x. */
int carekv_quantize(const void *x, int8_t *codes, void *scale, int64_t rows, int32_t D,
                    int32_t bits, int32_t group_size, int32_t dtype, void *stream);
/* dequantize (quantizer.py:67-82): codes*scale in fp32, cast to dtype. */
int carekv_dequantize(const int8_t *codes, const void *scale, void *out, int64_t rows, int32_t D,
                      int32_t group_size, int32_t dtype, void *stream);
/* pack_codes_2d / unpack_codes_2d (quantizer.py:364-383). */
int carekv_pack_codes(const int8_t *codes, uint8_t *packed, int64_t rows, int32_t D, int32_t bits,
                      void *stream);
int carekv_unpack_codes(const uint8_t *packed, int8_t *codes, int64_t rows, int32_t D, int32_t bits,
                        void *stream);
/* pack_4bit / unpack_4bit (residual_store.py:121-146) on `n` independent
 * blocks of `numel` fp32 values each (numel even). */
int carekv_pack_4bit(const float *x, uint8_t *packed, uint16_t *scale_f16, int64_t n, int32_t numel,
                     void *stream);
int carekv_unpack_4bit(const uint8_t *packed, const uint16_t *scale_f16, float *out, int64_t n,
                       int32_t numel, void *stream);

/* KIVI-style quantize-dequantize (kivi_helpers.py:35-59), in dtype:
 * _k: K [n][T][D], symmetric INT`bits` codes with a per-channel scale
 *     amax over T / qmax (quant_dequant_kivi_k);
 * _v: V [rows][D], per-token scale amax over D / qmax (quant_dequant_kivi_v).
 * out may alias the input. */
int carekv_kivi_quant_dequant_k(const void *K, void *out, int64_t n, int32_t T, int32_t D, int32_t bits,
                                int32_t dtype, void *stream);
int carekv_kivi_quant_dequant_v(const void *V, void *out, int64_t rows, int32_t D, int32_t bits,
                                int32_t dtype, void *stream);

/* ---- cache path ----------------------------------------------------------- */
/* Prefill store of `T` rows for sequences [seq_begin, seq_begin+seq_count)
 * of layer `layer`: allocates ceil(T/page_size) pages per kv head after the
 * pages already held, quantizes and packs rows, writes int8 page scales,
 * enumerates and keeps residual slots.  K, V: [seq_count][H][T][D] in
 * params->input_dtype.  sketch_proj: [k_channel_group][sketch_dim] fp32
 * (required when cfg->sketch_dim > 0).  Replaces layer.py:204-334. */
int carekv_prefill_store(const carekv_config_t *cfg, const carekv_cache_t *cache, int32_t layer,
                         const void *K, const void *V, int32_t T, int32_t seq_begin,
                         int32_t seq_count, const carekv_store_params_t *params,
                         const float *sketch_proj, void *stream);

/* Append one token per sequence to layer `layer` (decode): k, v
 * [seq_count][H][D] in params->input_dtype.  Opens a page when needed and,
 * when a page fills, re-runs the residual store on it as the reference does
 * (layer.py:1087-1146).  The page-full store runs only when may_fill_page
 * is nonzero; a caller that knows no sequence completes a page in this
 * call may pass 0 to skip those two launches.  A page needed beyond
 * max_pages is not written; the device sets bit 1 of cache->error_flag. */
int carekv_append(const carekv_config_t *cfg, const carekv_cache_t *cache, int32_t layer,
                  const void *k, const void *v, int32_t seq_begin, int32_t seq_count,
                  const carekv_store_params_t *params, const float *sketch_proj,
                  int32_t may_fill_page, void *stream);

/* ---- kv-head shards ------------------------------------------------------ */
/* An arena may hold a contiguous range of a model's kv heads: kv heads
 * [kvh_begin, kvh_begin + cfg->num_kv_heads) of a model with kvh_total kv
 * heads (each with cfg->num_heads / cfg->num_kv_heads query heads), as when
 * the kv heads of a layer are spread over GPUs (Mistral-7B: 8 kv heads, one
 * per GPU).  The _shard forms below take the model's full activation rows
 * -- K / V [seq_count][kvh_total][T][D], k / v [seq_count][kvh_total][D],
 * q / out [seq_count][kvh_total * QN][D] -- and read or write only this
 * shard's heads, so no caller-side gather or scatter is needed.  The plain
 * entry points are the shard {0, cfg->num_kv_heads}.  The work of a
 * (sequence, kv head) is independent of every other, so shards exchange
 * nothing (the reference's per (layer, kv head) slot pools and budgets,
 * attention.py:576). */
typedef struct carekv_shard {
    int32_t kvh_begin;   /* first model kv head held by the arena */
    int32_t kvh_total;   /* kv heads of the model's activation rows */
} carekv_shard_t;

int carekv_prefill_store_shard(const carekv_config_t *cfg, const carekv_cache_t *cache, int32_t layer,
                               const void *K, const void *V, int32_t T, int32_t seq_begin,
                               int32_t seq_count, const carekv_store_params_t *params,
                               const float *sketch_proj, const carekv_shard_t *shard, void *stream);
int carekv_append_shard(const carekv_config_t *cfg, const carekv_cache_t *cache, int32_t layer,
                        const void *k, const void *v, int32_t seq_begin, int32_t seq_count,
                        const carekv_store_params_t *params, const float *sketch_proj,
                        int32_t may_fill_page, const carekv_shard_t *shard, void *stream);

/* Workspace bytes carekv_decode_attention needs for `seq_count` sequences
 * holding at most `max_pages_used` pages per (layer, kv head). */
int carekv_decode_workspace_bytes(const carekv_config_t *cfg, int32_t seq_count,
                                  int32_t max_pages_used, size_t *bytes);

/* Decode attention for layer `layer`: base attention over the packed
 * pages plus the routed residual correction.  q, out: [seq_count][num_heads][D]
 * in `dtype`.  The workspace must hold carekv_decode_workspace_bytes.
 * sketch_proj ([k_channel_group][sketch_dim] fp32) is read only by the
 * sketch proxy score (params->kscore_live == 0).  Any read budget is served:
 * selections of more than 32 slots per query are applied in rounds.
 * Replaces CAREKVMultiHeadAttention.forward (attention.py:1042-1077) with
 * vectorized_joint_correction applied to each kv head's query group. */
int carekv_decode_attention(const carekv_config_t *cfg, const carekv_cache_t *cache, int32_t layer,
                            const void *q, void *out, int32_t dtype, int32_t seq_begin,
                            int32_t seq_count, int32_t max_pages_used,
                            const carekv_route_params_t *params, const float *sketch_proj,
                            void *workspace, size_t workspace_bytes, void *stream);

/* carekv_decode_attention on a kv-head shard (see carekv_shard_t): q / out
 * are the model's rows [seq_count][shard->kvh_total * QN][D]; the workspace
 * is sized for this arena's own kv heads. */
int carekv_decode_attention_shard(const carekv_config_t *cfg, const carekv_cache_t *cache, int32_t layer,
                                  const void *q, void *out, int32_t dtype, int32_t seq_begin,
                                  int32_t seq_count, int32_t max_pages_used,
                                  const carekv_route_params_t *params, const float *sketch_proj,
                                  void *workspace, size_t workspace_bytes, const carekv_shard_t *shard,
                                  void *stream);

/* Kernel launches one carekv_decode_attention call over `seq_count`
 * sequences issues: a split-K pass and a route kernel per batch chunk.  The
 * batch runs in CAREKV_ATTEND_CHUNKS (environment, 1 / 2 / 4, default 1)
 * chunks; with more than one they run on prioritised streams forked from the
 * caller's stream and joined back into it (events, so stream capture records
 * them), routing of one chunk overlapping the split-K pass of the next.  The
 * helper streams and
 * events belong to the calling host thread (one set per thread and device,
 * created by its first call outside stream capture; a thread whose first
 * call is captured runs that call unchunked), so several host threads may
 * call concurrently on one device, and one thread may capture while others
 * run uncaptured calls. */
int carekv_decode_attention_launches(const carekv_config_t *cfg, int32_t seq_count, int32_t *launches);

/* Decode attention for callers that cannot allocate device memory.
 *
 * No counterpart in the reference.  Same inputs, output and result as
 * carekv_decode_attention, but the scratch is a fixed array compiled into
 * this library (CAREKV_NOALLOC_MAX_BYTES per device, reserved on every GPU
 * that loads the library until the process exits) instead of a caller
 * workspace.  It is meant for callers that have no device allocator at hand
 * or may not use one while a step runs: a serving engine that owns all
 * device memory through its own pool, a host runtime binding this ABI with
 * no access to cudaMalloc, or a latency-bound loop that must avoid the
 * device synchronisation an allocation implies.
 *
 * The first call made while a device is current looks up that device's
 * array (cudaGetSymbolAddress) and caches the address; make that first call
 * before any stream capture.  A call whose scratch need
 * (carekv_decode_workspace_bytes) exceeds CAREKV_NOALLOC_MAX_BYTES returns
 * CAREKV_ERR_WORKSPACE without running anything.  All calls share the one
 * array: no part of it needs clearing between calls, but calls that may
 * overlap on the GPU race on it, so the caller must serialise them.  The call
 * allocates nothing.
 *
 * Which shapes fit: with S sequences, H kv heads, QN query heads per kv head,
 * P = max_pages_used and SK / SV slots per page, the scratch is about
 *   S*H*QN*P*(8*(SK+SV) + 64 + 64*SK) bytes
 * (selection readback and scores, logits, q . R_K of the stored K slots)
 * plus the split-K partials, S*H*splits*QN*(head_dim+2)*4 bytes.  Examples:
 * 32 sequences x 32 kv heads x 4096-token context (P = 264, SK = SV = 1,
 * QN = 1, Llama-2-7B shape) need 37.6 MiB and fit; 16 sequences x 8 kv
 * heads x 4 query heads x 32768 tokens (P = 2056, Mistral-7B shape) need
 * 147 MiB and are rejected, while one kv head of that batch (a shard of
 * one kv head per GPU) needs 19.1 MiB and fits. */
#define CAREKV_NOALLOC_MAX_BYTES ((size_t)64 << 20)
int carekv_decode_attention_noalloc(const carekv_config_t *cfg, const carekv_cache_t *cache,
                                    int32_t layer, const void *q, void *out, int32_t dtype,
                                    int32_t seq_begin, int32_t seq_count, int32_t max_pages_used,
                                    const carekv_route_params_t *params, const float *sketch_proj,
                                    void *stream);

/* Stored-slot correction of a prefill (CAREKV_PREFILL_MODE=carekv_stored):
 * for every prefill position t of cache sequence `seq` and every query head,
 * route over the slots the prefill just stored and add the correction to the
 * base output, as _apply_sparse_prefill_correction_stored (layer.py:458-637)
 * does with vectorized_joint_correction per kv head.  Inputs, with
 * P = max_pages_used and QN = num_heads / num_kv_heads:
 *   q       [n_pos][num_heads][D] post-RoPE queries in `dtype`
 *   logits  [n_pos][num_kv_heads][QN][P * 16] fp32 masked logits, token j of
 *           page p at p*16+j; read by the sketch proxy score only
 *           (params->kscore_live == 0), may be NULL otherwise
 *   row_max [n_pos][num_kv_heads][QN] fp32 maximum of each logit row (same
 *           condition)
 *   attn    [n_pos][num_kv_heads][QN][P * 16] fp32 attention weights of the
 *           (causally masked) prefill attention, laid out like logits
 *   attn_sum [n_pos][num_kv_heads][QN] fp32 row sums of attn, or NULL for 1
 *   o_base  [n_pos][num_kv_heads][QN][D] fp32 base output: the result where
 *           nothing is corrected, the start of the linear correction and
 *           of the sketch proxy's value distances
 *   o_exact [n_pos][num_kv_heads][QN][D] fp32 attn @ V in fp32, the start
 *           of the exact renormalisation a_new @ V, or NULL for o_base
 *   v_rows  [num_kv_heads][P * 16][D] fp32 base V rows the correction reads,
 *           or NULL for the cache's dequantised V
 *   v_pnorm [num_kv_heads][P] fp32 Frobenius norm of each page of v_rows, or
 *           NULL for the cache's page norms
 * out: [n_pos][num_heads][D] in `dtype`.  The workspace must hold
 * carekv_prefill_workspace_bytes(cfg, n_pos, max_pages_used).  The router
 * computes q . R_K from the slot payloads itself. */
int carekv_prefill_workspace_bytes(const carekv_config_t *cfg, int32_t n_pos, int32_t max_pages_used,
                                   size_t *bytes);
int carekv_prefill_correction(const carekv_config_t *cfg, const carekv_cache_t *cache, int32_t layer,
                              int32_t seq, int32_t n_pos, int32_t max_pages_used, const void *q,
                              const float *logits, const float *row_max, const float *attn,
                              const float *attn_sum, const float *o_base, const float *o_exact,
                              const float *v_rows, const float *v_pnorm, void *out,
                              int32_t dtype, const carekv_route_params_t *params,
                              const float *sketch_proj, void *workspace, size_t workspace_bytes,
                              void *stream);

/* Copy the device error flag to the host and clear it (synchronizes the
 * stream).  Returns CAREKV_OK when no device check tripped. */
int carekv_check_device_errors(const carekv_cache_t *cache, int32_t *flags_out, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* CAREKV_B200_H */
