// Route + correct kernel (K4 + K2) after every split-K pass: one CTA per
// (sequence, kv head, query head) runs route_body (route_body.cuh) -- the
// query heads of a GQA group route independently (per-query scores, budgets
// and top-k), so a group of QN heads takes QN CTAs in parallel.  The
// prefill correction keeps a group in one CTA.
#include "common.cuh"
#include "internal.h"
#include "decode_args.h"
#include "route_body.cuh"

namespace carekv {

// PF: prefill correction (caller attention weights, base V rows, one cache
// sequence for every row); the decode instantiation carries none of it.
// NW warps per CTA at 64 registers a thread: 4 (8 CTAs per SM) when the
// grid fills the GPU, 8 or 16 when it holds fewer CTAs than that (small
// batches, kv-head shards, long contexts with few sequences), so the
// per-CTA latency of a (sequence, kv head) spreads over more warps.
template <int QN, bool PF, int NW>
__global__ void __launch_bounds__(NW * 32, 32 / NW) route_kernel2(DecodeArgs a, int scores_in_smem) {
  __shared__ RouteSmem<QN, NW> sm;
  extern __shared__ float dyn[];
  route_body<QN, NW, PF>(a, blockIdx.x, sm, dyn, scores_in_smem);
}

template <int NW>
static cudaError_t launch_route_decode(DecodeArgs& a, cudaStream_t st, int n_bh, int qn, int NG) {
  const size_t sc_bytes = static_cast<size_t>(NG) * sizeof(float);
  const int in_smem = sc_bytes + sizeof(RouteSmem<1, NW>) <= 46 * 1024 ? 1 : 0;
  route_kernel2<1, false, NW><<<dim3(n_bh, qn), NW * 32, in_smem ? sc_bytes : 0, st>>>(a, in_smem);
  return cudaGetLastError();
}

template <int QN>
cudaError_t launch_route(DecodeArgs& a, cudaStream_t st, int n_bh) {
  constexpr int kSMs = 148;
  const int NG = a.p_used * (a.cfg.k_slots_per_page + a.cfg.v_slots_per_page);
  if (a.attn != nullptr) {
    const size_t sc_bytes = static_cast<size_t>(QN) * NG * sizeof(float);
    const int in_smem = sc_bytes + sizeof(RouteSmem<QN, 4>) <= 46 * 1024 ? 1 : 0;
    route_kernel2<QN, true, 4><<<n_bh, 4 * 32, in_smem ? sc_bytes : 0, st>>>(a, in_smem);
    return cudaGetLastError();
  }
  const int ctas = n_bh * QN;
  if (ctas <= 2 * kSMs) return launch_route_decode<16>(a, st, n_bh, QN, NG);
  if (ctas <= 4 * kSMs) return launch_route_decode<8>(a, st, n_bh, QN, NG);
  return launch_route_decode<4>(a, st, n_bh, QN, NG);
}

template cudaError_t launch_route<1>(DecodeArgs&, cudaStream_t, int);
template cudaError_t launch_route<2>(DecodeArgs&, cudaStream_t, int);
template cudaError_t launch_route<4>(DecodeArgs&, cudaStream_t, int);
template cudaError_t launch_route<8>(DecodeArgs&, cudaStream_t, int);

}  // namespace carekv
