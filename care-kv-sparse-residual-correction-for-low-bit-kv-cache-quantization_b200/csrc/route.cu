// Route + correct kernel (K4 + K2) after every split-K pass: one CTA of
// kRouteWarps warps per (sequence, kv head, query head) runs route_body
// (route_body.cuh) -- the query heads of a GQA group route independently
// (per-query scores, budgets and top-k), so a group of QN heads takes QN
// CTAs in parallel; small CTAs keep 8 of them resident per SM.  The prefill
// correction keeps a group in one CTA.
#include "common.cuh"
#include "internal.h"
#include "decode_args.h"
#include "route_body.cuh"

namespace carekv {

constexpr int kRouteWarps = 4;

// PF: prefill correction (caller attention weights, base V rows, one cache
// sequence for every row); the decode instantiation carries none of it.
template <int QN, bool PF>
__global__ void __launch_bounds__(kRouteWarps * 32, 8) route_kernel2(DecodeArgs a, int scores_in_smem) {
  __shared__ RouteSmem<QN, kRouteWarps> sm;
  extern __shared__ float dyn[];
  route_body<QN, kRouteWarps, PF>(a, blockIdx.x, sm, dyn, scores_in_smem);
}

template <int QN>
cudaError_t launch_route(DecodeArgs& a, cudaStream_t st, int n_bh) {
  const int NG = a.p_used * (a.cfg.k_slots_per_page + a.cfg.v_slots_per_page);
  if (a.attn != nullptr) {
    const size_t sc_bytes = static_cast<size_t>(QN) * NG * sizeof(float);
    const int in_smem = sc_bytes + sizeof(RouteSmem<QN, kRouteWarps>) <= 46 * 1024 ? 1 : 0;
    route_kernel2<QN, true><<<n_bh, kRouteWarps * 32, in_smem ? sc_bytes : 0, st>>>(a, in_smem);
  } else {
    const size_t sc_bytes = static_cast<size_t>(NG) * sizeof(float);
    const int in_smem = sc_bytes + sizeof(RouteSmem<1, kRouteWarps>) <= 46 * 1024 ? 1 : 0;
    route_kernel2<1, false><<<dim3(n_bh, QN), kRouteWarps * 32, in_smem ? sc_bytes : 0, st>>>(a, in_smem);
  }
  return cudaGetLastError();
}

template cudaError_t launch_route<1>(DecodeArgs&, cudaStream_t, int);
template cudaError_t launch_route<2>(DecodeArgs&, cudaStream_t, int);
template cudaError_t launch_route<4>(DecodeArgs&, cudaStream_t, int);
template cudaError_t launch_route<8>(DecodeArgs&, cudaStream_t, int);

}  // namespace carekv
