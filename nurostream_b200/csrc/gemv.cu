// ns_gemv: fused dequant-GEMV from GGUF bytes (batch 1..NS_MAX_TOKENS).
//
// Layout: each CTA owns a contiguous run of rows, walked in tiles of TR rows.
// A tile's bytes are one contiguous range of the weight buffer; thread 0
// streams tiles into a 3-stage shared-memory ring with 1-D bulk copies (the
// TMA engine, completion on an mbarrier), so ~2 tiles are in flight while the
// CTA decodes the third.  The activations are converted to fp32 once per CTA
// and kept in shared memory.  8 warps split a tile's rows R at a time; the 32
// lanes of a warp split each row's 32-element groups (qdot.cuh).
#include "qdot.cuh"

namespace ns {

constexpr int kGemvThreads = 256;
constexpr int kGemvStages = 3;
constexpr int kSmemBudget = 220 * 1024;
constexpr int kXG = 36;  // shared-memory floats per 32-element group of x

struct GemvArgs {
  const uint8_t* w;
  const uint8_t* w_end;
  int n_rows, K, rb, T;
  const void* x;
  int x_dtype;
  int64_t x_stride;
  void* y;
  int y_dtype;
  int64_t y_stride;
  int tile_rows;
  int stage_bytes;
};

template <int FMT, int NT, int R>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_kernel(GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int K = a.K, T = a.T;
  float* xs = reinterpret_cast<float*>(smem);
  // x in fp32, each 32-element group padded to kXG floats (lane g reads group g: distinct banks)
  const int xt = (K / 32) * kXG;  // floats per token
  uint8_t* stages = smem + (size_t)T * xt * 4;
  uint64_t* bars = reinterpret_cast<uint64_t*>(stages + kGemvStages * a.stage_bytes);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  // contiguous, balanced row range of this CTA
  const int r_begin = (int)((int64_t)a.n_rows * blockIdx.x / gridDim.x);
  const int r_end = (int)((int64_t)a.n_rows * (blockIdx.x + 1) / gridDim.x);
  const int n_tiles = (r_end - r_begin + a.tile_rows - 1) / a.tile_rows;

  auto tile_span = [&](int i) -> Span {
    int r0 = r_begin + i * a.tile_rows;
    int r1 = min(r0 + a.tile_rows, r_end);
    return Span{a.w + (int64_t)r0 * a.rb, a.w + (int64_t)r1 * a.rb};
  };
  auto issue = [&](int i) {
    uint64_t* bar = &bars[i % kGemvStages];
    Span s = tile_span(i);
    uintptr_t lo, hi;
    bulk_window(s, a.w, a.w_end, &lo, &hi);
    mbar_arrive_expect_tx(bar, hi > lo ? (uint32_t)(hi - lo) : 0u);
    issue_span(stages + (i % kGemvStages) * a.stage_bytes, s, a.w, a.w_end, bar);
  };

  if (tid == 0) {
    for (int s = 0; s < kGemvStages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
    for (int i = 0; i < kGemvStages && i < n_tiles; ++i) issue(i);
  }
  // activations -> fp32 shared memory (overlaps with the first copies)
  for (int i = tid; i < T * K; i += kGemvThreads) {
    int t = i / K, k = i - t * K;
    xs[t * xt + (k >> 5) * kXG + (k & 31)] = load_float(a.x, a.x_dtype, (int64_t)t * a.x_stride + k);
  }
  __syncthreads();

  const int ngroups = K / 32;
  for (int i = 0; i < n_tiles; ++i) {
    const int st = i % kGemvStages;
    uint8_t* buf = stages + st * a.stage_bytes;
    const Span s = tile_span(i);
    bool ok = mbar_wait_bounded(&bars[st], (uint32_t)((i / kGemvStages) & 1));
    if (span_has_ragged(s, a.w, a.w_end)) {
      if (warp == 0) copy_ragged(buf, s, a.w, a.w_end, lane);
      __syncthreads();
    }
    if (ok) {
      const int r0 = r_begin + i * a.tile_rows;
      const int nr = (int)((s.g1 - s.g0) / a.rb);
      const uint8_t* base = buf + (reinterpret_cast<uintptr_t>(s.g0) & 15);
      for (int rr = warp * R; rr < nr; rr += (kGemvThreads / 32) * R) {
        const uint8_t* rows[R];
        const int nrows = min(R, nr - rr);
#pragma unroll
        for (int r = 0; r < R; ++r) rows[r] = base + (int64_t)(rr + min(r, nrows - 1)) * a.rb;
        float acc[R][NT];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
          for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;
        int tok[NT];
#pragma unroll
        for (int t = 0; t < NT; ++t) tok[t] = t;
        dot_rows<FMT, NT, R, kXG>(rows, nrows, ngroups, lane, xs, xt, tok, T, acc);
#pragma unroll
        for (int r = 0; r < R; ++r) {
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            float v = warp_sum(acc[r][t]);
            if (lane == 0 && r < nrows && t < T)
              store_float(a.y, a.y_dtype, (int64_t)t * a.y_stride + r0 + rr + r, v);
          }
        }
      }
    }
    __syncthreads();  // stage st fully consumed
    if (tid == 0 && i + kGemvStages < n_tiles) issue(i + kGemvStages);
  }
}

template <int FMT, int NT, int R>
static int launch_gemv(const GemvArgs& a, int grid, size_t smem, cudaStream_t stream) {
  auto kern = gemv_kernel<FMT, NT, R>;
  NS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  kern<<<grid, kGemvThreads, smem, stream>>>(a);
  NS_CUDA_TRY(cudaGetLastError());
  return NS_OK;
}

template <int FMT>
static int dispatch_gemv_t(const GemvArgs& a, int grid, size_t smem, cudaStream_t stream) {
  if (a.T == 1) return launch_gemv<FMT, 1, 4>(a, grid, smem, stream);
  if (a.T == 2) return launch_gemv<FMT, 2, 4>(a, grid, smem, stream);
  if (a.T <= 4) return launch_gemv<FMT, 4, 2>(a, grid, smem, stream);
  return launch_gemv<FMT, 8, 2>(a, grid, smem, stream);
}

}  // namespace ns

extern "C" int ns_gemv(const uint8_t* w, size_t w_bytes, int ggml_type, int n_rows, int K, const void* x,
                       int x_dtype, int64_t x_stride, int T, void* y, int y_dtype, int64_t y_stride,
                       ns_stream_t stream) {
  using namespace ns;
  if (ggml_type != NS_GGML_MXFP4 && ggml_type != NS_GGML_Q8_0 && ggml_type != NS_GGML_Q4_K &&
      ggml_type != NS_GGML_Q6_K)
    return fail(NS_ERR_UNSUPPORTED, "ns_gemv: ggml type %d has no fused GEMV (MXFP4, Q8_0, Q4_K, Q6_K)",
                ggml_type);
  if (n_rows < 0 || K <= 0 || T < 1 || T > NS_MAX_TOKENS)
    return fail(NS_ERR_INVALID, "ns_gemv: bad shape n_rows=%d K=%d T=%d (T must be 1..%d)", n_rows, K, T,
                NS_MAX_TOKENS);
  if (!float_type_ok(x_dtype) || !float_type_ok(y_dtype))
    return fail(NS_ERR_INVALID, "ns_gemv: bad float type x=%d y=%d", x_dtype, y_dtype);
  const int64_t rb = row_bytes_of(ggml_type, K);
  if (rb < 0) return fail(NS_ERR_INVALID, "ns_gemv: K=%d is not a whole number of blocks", K);
  if (n_rows == 0) return NS_OK;
  if (!w || !x || !y) return fail(NS_ERR_INVALID, "ns_gemv: null pointer");
  if ((uint64_t)n_rows * (uint64_t)rb > w_bytes)
    return fail(NS_ERR_SIZE, "ns_gemv: weight buffer has %zu bytes, %d rows need %lld", w_bytes, n_rows,
                (long long)(n_rows * rb));
  if (x_stride < K || y_stride < n_rows)
    return fail(NS_ERR_INVALID, "ns_gemv: strides too small (x %lld < %d or y %lld < %d)",
                (long long)x_stride, K, (long long)y_stride, n_rows);

  int nsm = 0;
  int st = num_sms(&nsm);
  if (st) return st;
  const size_t x_bytes = (size_t)T * (K / 32) * kXG * 4;
  if (x_bytes + kGemvStages * (rb + 64) + 64 > (size_t)kSmemBudget)
    return fail(NS_ERR_UNSUPPORTED, "ns_gemv: T*K=%d activations plus a %lld-byte row exceed shared memory",
                T * K, (long long)rb);
  int stage_bytes = (int)std::min<size_t>(48 * 1024, ((kSmemBudget - x_bytes - 64) / kGemvStages) & ~size_t(15));
  int tr_max = (int)((stage_bytes - 64) / rb);
  int per_cta = (n_rows + nsm - 1) / nsm;
  int tile_rows = std::max(1, std::min(tr_max, per_cta));
  int grid = std::min(nsm, (n_rows + tile_rows - 1) / tile_rows);
  size_t smem = x_bytes + (size_t)kGemvStages * stage_bytes + kGemvStages * 8;

  GemvArgs a{w, w + w_bytes, n_rows, K, (int)rb, T, x, x_dtype, x_stride, y, y_dtype, y_stride, tile_rows,
             stage_bytes};
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (ggml_type) {
    case NS_GGML_MXFP4: return dispatch_gemv_t<NS_GGML_MXFP4>(a, grid, smem, s);
    case NS_GGML_Q8_0: return dispatch_gemv_t<NS_GGML_Q8_0>(a, grid, smem, s);
    case NS_GGML_Q4_K: return dispatch_gemv_t<NS_GGML_Q4_K>(a, grid, smem, s);
    default: return dispatch_gemv_t<NS_GGML_Q6_K>(a, grid, smem, s);
  }
}
