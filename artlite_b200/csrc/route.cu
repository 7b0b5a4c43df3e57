// Routing: one warp per token, top-k by rounds of a warp arg-max over 64-bit ordered keys, softmax / sigmoid weights
// over the k in double, normalised in numpy's pairwise order.
//
// Semantics follow artlite::moe_route (csrc/artlite/moe_host.cpp:45-73 route_rows_scalar, :98-174
// route_rows_avx512, :216-239 route_rows / moe_route):
//   key(l, x) = (bits(l + 0) flipped to an unsigned order) << 32 | ~x  (ties to the lower id, -0 == +0, :95-96);
//   e_j = e^(l_j - l_0) in double; on the reference's vector-path shapes (k <= 16, per_col % 16 == 0, E <= 512) rows
//   with k == 8, softmax and no NaN take its degree-12 Taylor exp_nonpos (:115-130, restated below from that
//   source), every other row exp() (the reference's std::exp); sigmoid: 1 / (1 + e^-l) with the sum clamped at 2^-14;
//   the sum in numpy's pairwise order (row_sum, :64-79); w_j = float(e_j / sum).
// The GPU's float add returns a canonical NaN where x86's keeps the operand's sign and payload, so the key is built
// from the bits directly: -0 -> +0, a NaN quietened with its sign kept (what addss(l, 0) gives).
#include "common.cuh"
#include "kernels.cuh"
#include "route.cuh"

namespace artlite {

template <int J>
__global__ void __launch_bounds__(256) route_kernel(RouteArgs a) {
  griddep_wait();
  griddep_launch();
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t < a.n) route_row<J>(a, t, threadIdx.x & 31);
}

int launch_route(const RouteArgs& a, cudaStream_t st) {
  if (a.n == 0) return ARTLITE_OK;
  const int warps = 8;
  const unsigned grid = (unsigned)cdiv(a.n, warps);
  const int J = (a.E + 31) / 32;
  const dim3 g(grid), b(warps * 32);
  if (J <= 1) return launch_pdl(route_kernel<1>, g, b, 0, st, a);
  if (J <= 2) return launch_pdl(route_kernel<2>, g, b, 0, st, a);
  if (J <= 4) return launch_pdl(route_kernel<4>, g, b, 0, st, a);
  if (J <= 8) return launch_pdl(route_kernel<8>, g, b, 0, st, a);
  if (J <= 16) return launch_pdl(route_kernel<16>, g, b, 0, st, a);
  return launch_pdl(route_kernel<32>, g, b, 0, st, a);
}

int check_route_args(int64_t n, int per_col, int E, int k) {
  // the reference's own check (moe_host.cpp:188), then this build's limits
  AL_CHECK(per_col > 0 && k >= 1 && k <= E && E % per_col == 0, ARTLITE_EINVAL, "moe_route: k %d of E %d (%d per column)",
           k, E, per_col);
  AL_CHECK(E <= 1024 && k <= 32, ARTLITE_EUNSUPPORTED, "moe_route: E %d k %d (this build: E <= 1024, k <= 32)", E, k);
  AL_CHECK(n >= 0, ARTLITE_EINVAL, "moe_route: n %lld", (long long)n);
  return ARTLITE_OK;
}

}  // namespace artlite
