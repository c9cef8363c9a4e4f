// Decode attention over the packed cache (kernels K3, K4 and K2).
//
// K3 split-K pass (decode_narrow.cu, decode_fast.cu, decode_generic.cu):
//   each CTA streams a range of pages of one (sequence, kv head),
//   dequantizes K and V rows to their fp16 values, computes the logits of
//   the kv head's query group, keeps an online softmax and the weighted V
//   sum, writes the logits (the router needs the normalised weights of every
//   token) and q . R_K of the stored K slots to the workspace, and one
//   (m, l, O) partial per CTA; this file plans and launches it.
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
#include "decode_args.h"
#include "ptx.cuh"
#include <algorithm>
#include <cstdlib>

namespace carekv {

// ─────────────────────────── host launch ───────────────────────────
struct SplitPlan {
  int pps, n_splits;
};

// Pages per split.  A CTA costs its pages plus a fixed overhead (query
// operands, pipeline fill, partial merge; about kCtaOverheadPages pages of
// streaming, fitted to measured call times), and the pass takes as many
// waves as its CTAs fill `slots` resident CTAs over the 148 SMs:
//   cost(ns) = waves(ns) * (pages per CTA + kCtaOverheadPages),
// minimised over ns with at least 64 pages per CTA (16 per warp, enough to
// fill the staging pipeline); fewer splits win ties.  A large batch (1024
// (sequence, kv head) pairs of 264 pages) then runs one split, a small one
// (128 pairs) four.
constexpr int kCtaOverheadPages = 32;
inline SplitPlan split_plan(int n_bh, int p_used, int slots) {
  int best_ns = 1;
  long long best = -1;
  for (int ns = 1; ns <= 32; ++ns) {
    const int pps = (p_used + ns - 1) / ns;
    if (ns > 1 && pps < 64) break;
    const long long total = static_cast<long long>(n_bh) * ns;
    const long long waves = (total + slots - 1) / slots;
    const long long cost = waves * (pps + kCtaOverheadPages);
    if (best < 0 || cost < best) {
      best = cost;
      best_ns = ns;
    }
  }
  SplitPlan sp;
  sp.pps = (p_used + best_ns - 1) / best_ns;
  sp.pps = max(sp.pps, 1);
  sp.n_splits = max(1, (p_used + sp.pps - 1) / sp.pps);
  return sp;
}

static inline int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }
// Entries per query of the selection readback: the count, then room for
// every slot of the grid (a selection has no other upper bound).
static inline int64_t sel_stride(const carekv_config_t& c, int p_used) {
  return 1 + static_cast<int64_t>(p_used) * (c.k_slots_per_page + c.v_slots_per_page);
}

// Split-K pass chosen for a layout.  NARROW: INT3 or INT4 / int8 scales with at most
// 4 query heads per kv head (decode_narrow.cu, 4 CTAs per SM); WIDE: INT3 with
// 8 query heads (decode_fast.cu, 2 CTAs per SM); both also compute q . R_K of
// the stored K slots.  GENERIC: every other layout (decode_generic.cu, which
// computes them too).
enum class Pass { GENERIC, WIDE, NARROW };
inline Pass choose_pass(const carekv_config_t& c) {
  const int D = c.head_dim;
  const bool tiled = c.base_kind == CAREKV_BASE_UNIFORM && c.scale_mode == CAREKV_SCALE_INT8 && (D == 64 || D == 128) &&
                     c.group_size % (D / 4) == 0 && c.group_size % (D / 8) == 0 && c.page_size == kPage;
  const int qn = c.num_heads / c.num_kv_heads;
  if (tiled && qn <= 4 && (c.base_bits == 3 || c.base_bits == 4)) return Pass::NARROW;
  if (tiled && c.base_bits == 3) return Pass::WIDE;
  return Pass::GENERIC;
}
inline int pass_slots(Pass p) { return p == Pass::NARROW ? 4 * 148 : 2 * 148; }

namespace {
int attend_chunks();
}
// Sequences per chunk of a decode attention call (see decode_attention).
inline int chunk_size(int seq_count) {
  const int chunks = std::max(1, std::min(attend_chunks(), seq_count));
  return (seq_count + chunks - 1) / chunks;
}

// Workspace regions, each 256-byte aligned: selection readback, scores,
// logits, split partials m / l / O, and (narrow and wide passes) q . R_K
// per K slot.
// The split plan is the one of a chunk (chunk_size sequences).
struct WsLayout {
  int64_t sel, scores, S, pm, pl, po, kw, total;
};
inline WsLayout ws_layout(const carekv_config_t& c, int seq_count, int p_used) {
  const int64_t qn = c.num_heads / c.num_kv_heads;
  const int64_t n_bh = static_cast<int64_t>(seq_count) * c.num_kv_heads;
  const Pass pass = choose_pass(c);
  const SplitPlan sp = split_plan(chunk_size(seq_count) * c.num_kv_heads, p_used, pass_slots(pass));
  WsLayout w;
  int64_t o = 0;
  w.sel = o;    o = align256(o + n_bh * qn * sel_stride(c, p_used) * 4);
  w.scores = o; o = align256(o + n_bh * qn * static_cast<int64_t>(p_used) * (c.k_slots_per_page + c.v_slots_per_page) * 4);
  w.S = o;      o = align256(o + n_bh * qn * static_cast<int64_t>(p_used) * kPage * 4);
  w.pm = o;     o = align256(o + n_bh * sp.n_splits * qn * 4);
  w.pl = o;     o = align256(o + n_bh * sp.n_splits * qn * 4);
  w.po = o;     o = align256(o + n_bh * sp.n_splits * qn * static_cast<int64_t>(c.head_dim) * 4);
  w.kw = o;
  o = align256(o + n_bh * qn * static_cast<int64_t>(p_used) * c.k_slots_per_page * kPage * 4);
  w.total = o;
  return w;
}

size_t workspace_bytes(const carekv_config_t& c, int seq_count, int p_used) {
  return static_cast<size_t>(ws_layout(c, seq_count, p_used).total);
}

// The prefill correction reads its logits and partials from the caller:
// only the selection readback and the scores live in the workspace.
size_t prefill_workspace_bytes(const carekv_config_t& c, int n_pos, int p_used) {
  return static_cast<size_t>(ws_layout(c, n_pos, p_used).S);
}

template <int QN>
static cudaError_t launch_qn(DecodeArgs& a, cudaStream_t st, int n_bh) {
  cudaError_t e;
  const Pass pass = a.force_generic ? Pass::GENERIC : choose_pass(a.cfg);
  if (pass == Pass::NARROW) {
    if constexpr (QN <= 4) {
      e = a.cfg.head_dim == 64 ? launch_decode_narrow<QN, 64>(a, st, n_bh)
                               : launch_decode_narrow<QN, 128>(a, st, n_bh);
    } else {
      return cudaErrorInvalidValue;
    }
  } else if (pass == Pass::WIDE) {
    e = a.cfg.head_dim == 64 ? launch_decode_partial_int3<QN, 64>(a, st, n_bh)
                             : launch_decode_partial_int3<QN, 128>(a, st, n_bh);
  } else {
    e = launch_decode_generic<QN>(a, st, n_bh);
  }
  if (e != cudaSuccess) return e;
  return launch_route<QN>(a, st, n_bh);
}

// Batch chunking of decode attention (optional; one chunk by default).  The
// batch may be cut into `chunks` ranges of sequences that run on separate
// streams: chunk c (c < chunks - 1) on an internal stream of higher priority
// than chunk c + 1, the last chunk on the caller's stream, so routing a
// chunk overlaps the split-K pass of the later chunks.  With the split-K
// pass at its current rate one chunk is faster at the benchmark shape (227
// vs 235 us per call at 32 sequences x 32 kv heads x 4096 tokens): the
// chunks' narrower grids cost more than the overlap gains.  Every chunk
// uses the split plan of one chunk and its slice of the one workspace layout
// (all regions are indexed by (sequence, kv head)), so the workspace size
// and the selection readback do not depend on the chunking.
// Fork and join go through events, which stream capture records as graph
// edges.  CAREKV_ATTEND_CHUNKS (1, 2 or 4; default 1) sets the count.
// The helper streams and events belong to the calling host thread (one set
// per device and thread), so concurrent calls from several threads, or a
// capture on one thread while another thread runs uncaptured calls, never
// share an event or a stream.
namespace {
constexpr int kMaxDev = 64, kMaxChunks = 4;
struct ChunkStreams {
  bool ready = false, failed = false;
  cudaStream_t st[kMaxChunks - 1] = {};
  cudaEvent_t fork = nullptr, join[kMaxChunks - 1] = {};
  // release whatever exists (a partial set after a failed creation, or the
  // whole set when the thread exits; errors after runtime teardown are moot)
  void release() {
    for (int i = 0; i < kMaxChunks - 1; ++i) {
      if (st[i]) (void)cudaStreamDestroy(st[i]);
      if (join[i]) (void)cudaEventDestroy(join[i]);
      st[i] = nullptr;
      join[i] = nullptr;
    }
    if (fork) (void)cudaEventDestroy(fork);
    fork = nullptr;
    ready = false;
  }
  ~ChunkStreams() {
    if (ready) release();
  }
};
thread_local ChunkStreams t_chunk[kMaxDev];

int attend_chunks() {
  static const int n = [] {
    const char* e = std::getenv("CAREKV_ATTEND_CHUNKS");
    const int v = e ? std::atoi(e) : 1;
    return v == 1 || v == 2 || v == 4 ? v : 1;
  }();
  return n;
}

// This thread's streams and events of the current device, created on first
// use outside stream capture; null while they do not exist (the caller then
// runs unchunked).  A creation that fails part-way releases what it made and
// leaves this thread on the device unchunked from then on.
ChunkStreams* chunk_streams(cudaStream_t caller) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return nullptr;
  ChunkStreams& cs = t_chunk[dev];
  if (cs.ready) return &cs;
  if (cs.failed) return nullptr;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(caller, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) return nullptr;
  int least = 0, greatest = 0;
  bool ok = cudaDeviceGetStreamPriorityRange(&least, &greatest) == cudaSuccess;
  for (int i = 0; ok && i < kMaxChunks - 1; ++i) {
    // chunk 0 gets the greatest priority, later chunks step down towards the caller's
    const int prio = std::min(least, greatest + i);
    ok = cudaStreamCreateWithPriority(&cs.st[i], cudaStreamNonBlocking, prio) == cudaSuccess &&
         cudaEventCreateWithFlags(&cs.join[i], cudaEventDisableTiming) == cudaSuccess;
  }
  ok = ok && cudaEventCreateWithFlags(&cs.fork, cudaEventDisableTiming) == cudaSuccess;
  if (!ok) {
    cs.release();
    cs.failed = true;
    (void)cudaGetLastError();   // the failure is handled here, not by the next launch check
    return nullptr;
  }
  cs.ready = true;
  return &cs;
}
}  // namespace

void prepare_decode_streams() { (void)chunk_streams(nullptr); }

int decode_attention_chunks(int seq_count) {
  if (seq_count <= 0) return 0;
  const int per = chunk_size(seq_count);
  return (seq_count + per - 1) / per;
}

int decode_attention(const carekv_config_t& cfg, const carekv_cache_t& cache, int layer, const void* q,
                     void* out, int dtype, int seq_begin, int seq_count, int p_used,
                     const carekv_route_params_t& rp, void* ws, size_t ws_bytes, const float* sketch_proj,
                     int act_heads, cudaStream_t st) {
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
  a.act_heads = act_heads;
  const int H = cfg.num_kv_heads;
  const SplitPlan sp = split_plan(chunk_size(seq_count) * H, p_used, pass_slots(choose_pass(cfg)));
  a.pps = sp.pps;
  a.n_splits = sp.n_splits;
  a.p_used = p_used;
  a.sf = static_cast<float>(1.0 / std::sqrt(static_cast<double>(cfg.head_dim)));
  a.sqrt_d = static_cast<float>(std::sqrt(static_cast<double>(cfg.head_dim)));
  // workspace: selection readback and scores first (their offsets do not
  // depend on the split plan), then logits and split partials
  const WsLayout wl = ws_layout(cfg, seq_count, p_used);
  char* w = static_cast<char*>(ws);
  a.sel_out = reinterpret_cast<int*>(w + wl.sel);
  a.sel_stride = static_cast<int>(sel_stride(cfg, p_used));
  a.scores = reinterpret_cast<float*>(w + wl.scores);
  a.S = reinterpret_cast<float*>(w + wl.S);
  a.pm = reinterpret_cast<float*>(w + wl.pm);
  a.pl = reinterpret_cast<float*>(w + wl.pl);
  a.po = reinterpret_cast<float*>(w + wl.po);
  // q . R_K is precomputed by the split-K pass whenever live
  // combined_kvscore scoring may read it: K slots stored and K residuals
  // part of the route
  const bool live_k = rp.kind != CAREKV_KIND_NONE && rp.kind != CAREKV_KIND_V && rp.kscore_live &&
                      cfg.k_slots_per_page > 0;
  a.kw = live_k ? reinterpret_cast<float*>(w + wl.kw) : nullptr;
  a.s_perm = 0;
  a.dq_keys[0] = i3_key2(0, 0);
  a.dq_keys[1] = i3_key2(3, 3);
  a.dq_keys[2] = i3_key2(6, 6);
  a.dq_keys[3] = 0x64086408u;
  a.dq_keys[4] = 0x54805480u;
  a.dq_keys[5] = i3_key2(1, 0);
  a.dq_keys[6] = i3_key2(4, 3);
  a.dq_keys[7] = i3_key2(7, 6);
  a.dq_keys[8] = i3_key2(2, 2);
  a.dq_keys[9] = i3_key2(1, 1);
  a.dq_keys[10] = i3_key2(4, 4);
  a.dq_keys[11] = i3_key2(7, 7);
  a.dq_keys[12] = i3_key2(5, 5);
  a.sketch_proj = sketch_proj;
  a.rp = rp;
  a.force_generic = 0;
  a.seq_fixed = -1;
  a.attn = nullptr;
  a.o_exact = nullptr;
  a.v_rows = nullptr;
  a.v_pnorm = nullptr;
  if (a.qn != 1 && a.qn != 2 && a.qn != 4 && a.qn != 8) return CAREKV_ERR_UNSUPPORTED;

  const int per = chunk_size(seq_count);
  int chunks = (seq_count + per - 1) / per;
  ChunkStreams* cs = chunks > 1 ? chunk_streams(st) : nullptr;
  // without the streams (first call under capture) the chunks run in order on
  // the caller's stream: same plan, same workspace slices, no overlap

  if (cs && cudaEventRecord(cs->fork, st) != cudaSuccess) return CAREKV_ERR_CUDA;
  const int64_t qn = a.qn, D = cfg.head_dim, NGs = static_cast<int64_t>(p_used) * (cfg.k_slots_per_page + cfg.v_slots_per_page);
  const int64_t es = dtype == CAREKV_F32 ? 4 : 2;
  for (int c = 0; c < chunks; ++c) {
    const int s0 = c * per, n = std::min(per, seq_count - s0);
    const int64_t bh0 = static_cast<int64_t>(s0) * H;
    DecodeArgs ac = a;
    ac.seq_begin = seq_begin + s0;
    ac.q = static_cast<const char*>(q) + static_cast<int64_t>(s0) * act_heads * D * es;
    ac.out = static_cast<char*>(out) + static_cast<int64_t>(s0) * act_heads * D * es;
    ac.sel_out = a.sel_out + bh0 * qn * a.sel_stride;
    ac.scores = a.scores + bh0 * qn * NGs;
    ac.S = a.S + bh0 * qn * p_used * kPage;
    ac.pm = a.pm + bh0 * a.n_splits * qn;
    ac.pl = a.pl + bh0 * a.n_splits * qn;
    ac.po = a.po + bh0 * a.n_splits * qn * D;
    if (a.kw) ac.kw = a.kw + bh0 * qn * p_used * cfg.k_slots_per_page * kPage;
    cudaStream_t sc = st;
    if (cs && c < chunks - 1) {
      sc = cs->st[c];
      if (cudaStreamWaitEvent(sc, cs->fork, 0) != cudaSuccess) return CAREKV_ERR_CUDA;
    }
    cudaError_t e;
    switch (a.qn) {
      case 1: e = launch_qn<1>(ac, sc, n * H); break;
      case 2: e = launch_qn<2>(ac, sc, n * H); break;
      case 4: e = launch_qn<4>(ac, sc, n * H); break;
      default: e = launch_qn<8>(ac, sc, n * H); break;
    }
    if (e != cudaSuccess) return CAREKV_ERR_CUDA;
    if (cs && c < chunks - 1) {
      if (cudaEventRecord(cs->join[c], sc) != cudaSuccess) return CAREKV_ERR_CUDA;
    }
  }
  for (int c = 0; cs && c < chunks - 1; ++c)
    if (cudaStreamWaitEvent(st, cs->join[c], 0) != cudaSuccess) return CAREKV_ERR_CUDA;
  return CAREKV_OK;
}

// Stored-slot prefill correction (layer.py:458-637 with the vectorized
// router, attention.py:576-957): the route kernel over n_pos x H grid rows,
// row (t, h) holding the QN query heads of kv head h at prefill position t.
// The caller supplies the attention weights A (causally masked, as the
// prefill attention produced them) with their row sums, the masked logits
// and their row maxima (read by the sketch proxy score only), the base
// output O and sum_t A V (the exact renormalisation's starting point), and
// optionally the prefill's base V rows and their page norms.
int prefill_correction(const carekv_config_t& cfg, const carekv_cache_t& cache, int layer, int seq, int n_pos,
                       int p_used, const void* q, const float* logits, const float* row_max, const float* A,
                       const float* A_sum, const float* O, const float* O_exact, const float* v_rows,
                       const float* v_pnorm, void* out, int dtype, const carekv_route_params_t& rp,
                       const float* sketch_proj, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (ws_bytes < prefill_workspace_bytes(cfg, n_pos, p_used)) return CAREKV_ERR_WORKSPACE;
  DecodeArgs a{};
  a.cfg = cfg;
  a.cache = cache;
  a.layer = layer;
  a.q = q;
  a.out = out;
  a.dt = dtype;
  a.seq_begin = 0;
  a.qn = cfg.num_heads / cfg.num_kv_heads;
  a.act_heads = cfg.num_heads;
  a.pps = p_used;
  a.n_splits = 0;
  a.p_used = p_used;
  a.sf = static_cast<float>(1.0 / std::sqrt(static_cast<double>(cfg.head_dim)));
  a.sqrt_d = static_cast<float>(std::sqrt(static_cast<double>(cfg.head_dim)));
  const WsLayout wl = ws_layout(cfg, n_pos, p_used);
  char* w = static_cast<char*>(ws);
  a.sel_out = reinterpret_cast<int*>(w + wl.sel);
  a.sel_stride = static_cast<int>(sel_stride(cfg, p_used));
  a.scores = reinterpret_cast<float*>(w + wl.scores);
  a.S = const_cast<float*>(logits);
  a.pm = const_cast<float*>(row_max);
  a.po = const_cast<float*>(O);
  a.attn = A;
  a.pl = const_cast<float*>(A_sum);
  a.o_exact = O_exact;
  a.sketch_proj = sketch_proj;
  a.kw = nullptr;
  a.s_perm = 0;
  a.rp = rp;
  a.seq_fixed = seq;
  a.v_rows = v_rows;
  a.v_pnorm = v_pnorm;
  const int n_bh = n_pos * cfg.num_kv_heads;
  cudaError_t e;
  switch (a.qn) {
    case 1: e = launch_route<1>(a, st, n_bh); break;
    case 2: e = launch_route<2>(a, st, n_bh); break;
    case 4: e = launch_route<4>(a, st, n_bh); break;
    case 8: e = launch_route<8>(a, st, n_bh); break;
    default: return CAREKV_ERR_UNSUPPORTED;
  }
  return e == cudaSuccess ? CAREKV_OK : CAREKV_ERR_CUDA;
}

}  // namespace carekv
