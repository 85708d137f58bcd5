// ns_dense_gemv: batch-1 projection with bf16 weights, fp32 activations and fp32 accumulation,
// with the RMSNorm in front of it and the bias / residual add behind it fused into the one launch.
//
// It stands in for the reference's float-weight projections: Qwen3Model._linear's `x @ W.T`
// (neurostream/model/qwen3.py:169-194) and GptOssModel._biased_linear (gpt_oss.py:97-99), with
// rms_norm (neurostream/compute/ops.py:14-20) and the residual `x + ...` of _attention_block
// (gpt_oss.py:101-114) folded in.  Up to NS_DENSE_MAX_SEG weight matrices with the same K form one
// concatenated row space (q, k and v of an attention block in one launch).
//
// The work is HBM-bound byte streaming: one FMA per 2 weight bytes.  Layout:
//  - one CTA per SM owns a contiguous, balanced run of rows, walked in tiles of kDenseTileRows rows;
//  - a producer warp streams each tile (one contiguous byte range per segment it touches) into a
//    ring of shared-memory stages with 1-D bulk copies (TMA engine, completion on an mbarrier);
//  - the 8 compute warps split K: thread t owns the 16-byte chunks t, t + 256, ... of every row, so
//    its slice of the (normalised) activations lives in registers for the whole launch and each
//    weight byte is read from shared memory exactly once;
//  - a tile's 8 row sums meet by a butterfly that halves the rows per step (9 shuffles for 8 rows),
//    then across warps in shared memory, in a fixed order (deterministic).
// Programmatic dependent launch: the weights never depend on an earlier kernel, so the producer
// fills the whole ring before griddepcontrol.wait; on an SM freed by the previous kernel the weight
// stream starts while that kernel's last CTAs finish.  Only x, norm_w, the biases and the residual
// are read after the wait.  The kernel lets its dependents launch only after its own wait, which
// keeps the stream's chain invariant: when a kernel starts, the kernel two places before it in the
// stream has completed.

namespace ns {

constexpr int kDenseWarps = 8;                        // compute warps
constexpr int kDenseThreads = (kDenseWarps + 1) * 32;  // + one producer warp
constexpr int kDenseTileRows = 8;
constexpr int kDenseMaxStages = 8;
#ifndef NS_DENSE_SMEM_KB
#define NS_DENSE_SMEM_KB 220
#endif
constexpr int kDenseSmemBudget = NS_DENSE_SMEM_KB * 1024;
constexpr int kDensePreRows = 1024;  // rows per CTA whose bias / residual are staged in shared memory

struct DenseArgs {
  ns_dense_gemv_t p;
  int total_rows;
  int seg_start[NS_DENSE_MAX_SEG + 1];  // first row of each segment in the concatenated row space
  int stages;
  int stage_bytes;
  int tile_rows;  // rows per stage, <= kDenseTileRows (fewer for wide K, so that 2+ stages fit)
  int pre;        // stage the CTA's biases / residuals (its rows fit kDensePreRows and some are given)
};

// Sum of 8 per-lane values across a warp, one row per lane group: after the butterfly, lane l
// holds the warp total of row ((l >> 4) & 1) * 4 + ((l >> 3) & 1) * 2 + ((l >> 2) & 1).
__device__ __forceinline__ float reduce8_rows(float (&v)[8], int lane) {
  const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
  float h[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float send = b4 ? v[i] : v[i + 4];
    const float keep = b4 ? v[i + 4] : v[i];
    h[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
  float q[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float send = b3 ? h[i] : h[i + 2];
    const float keep = b3 ? h[i + 2] : h[i];
    q[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  float r;
  {
    const float send = b2 ? q[0] : q[1];
    const float keep = b2 ? q[1] : q[0];
    r = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  r += __shfl_xor_sync(0xffffffffu, r, 2);
  r += __shfl_xor_sync(0xffffffffu, r, 1);
  return r;
}

// Barrier among the first nthreads threads (whole warps) that also ORs a predicate over them.
__device__ __forceinline__ bool named_sync_or(int id, int nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ int dense_row_of(int lane) {
  return ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
}

// NCH: 16-byte chunks of a row per compute thread (ceil(K / 8 / 256)).
template <int NCH>
__global__ void __launch_bounds__(kDenseThreads, 1) dense_gemv_kernel(DenseArgs a) {
  extern __shared__ __align__(128) uint8_t dense_smem[];
  const int nst = a.stages, K = a.p.K;
  const int row_bytes = K * 2;
  uint8_t* stages = dense_smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(dense_smem + (size_t)nst * a.stage_bytes);
  uint64_t* empty = full + kDenseMaxStages;
  float* red = reinterpret_cast<float*>(empty + kDenseMaxStages);  // [2][warp][row]
  float* ssq = red + 2 * kDenseWarps * kDenseTileRows;              // [warp]
  float* pre_b = ssq + kDenseWarps;                                  // [row - r_begin]: bias (0 if none)
  float* pre_r = pre_b + kDensePreRows;                              // [row - r_begin]: residual (0 if none)
  __shared__ int s_issued;              // tiles the producer issued (fewer only when a wait ran out)
  __shared__ volatile int s_prod_done;  // the producer has left its loop

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r_begin = (int)((int64_t)a.total_rows * blockIdx.x / gridDim.x);
  const int r_end = (int)((int64_t)a.total_rows * (blockIdx.x + 1) / gridDim.x);
  const int tr = a.tile_rows;
  const int n_tiles = (r_end - r_begin + tr - 1) / tr;

  if (tid == 0) {
    s_issued = 0;
    s_prod_done = 0;
    for (int s = 0; s < nst; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kDenseWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kDenseWarps) {
    // ---- producer: static weights only, so the first stages go out before the wait
    if (lane == 0) {
      int i = 0;
      bool hinted = false;
      for (; i < n_tiles; ++i) {
        if (i == nst && !hinted) {  // the ring is full: the later kernels' weights next (L2 hint)
          l2_prefetch_share(a.p.l2, blockIdx.x, gridDim.x);
          hinted = true;
        }
        const int slot = i % nst;
        // a wait that runs out means the compute warps gave up on an earlier tile: issue no more
        if (i >= nst && !mbar_wait_bounded(&empty[slot], (uint32_t)((i / nst - 1) & 1))) break;
        const int r0 = r_begin + i * tr, r1 = min(r0 + tr, r_end);
        mbar_arrive_expect_tx(&full[slot], (uint32_t)((r1 - r0) * row_bytes));
        uint8_t* dst = stages + (size_t)slot * a.stage_bytes;
        for (int s = 0; s < a.p.n_seg; ++s) {
          const int lo = max(r0, a.seg_start[s]), hi = min(r1, a.seg_start[s + 1]);
          if (lo >= hi) continue;
          const uint8_t* src =
              reinterpret_cast<const uint8_t*>(a.p.seg[s].w) + (int64_t)(lo - a.seg_start[s]) * row_bytes;
          uint32_t left = (uint32_t)((hi - lo) * row_bytes), off = (uint32_t)((lo - r0) * row_bytes);
          while (left > 0) {  // pieces of <= 16 KB: several copies in flight per stage
            const uint32_t n = min(left, 16384u);
            bulk_g2s(dst + off, src, n, &full[slot]);
            src += n;
            off += n;
            left -= n;
          }
        }
      }
      if (!hinted) l2_prefetch_share(a.p.l2, blockIdx.x, gridDim.x);
      s_issued = i;
      __threadfence_block();
      s_prod_done = 1;
    }
    return;
  }

  // ---- compute warps: activations after the previous kernel has completed
  griddep_wait();
  const float* x = a.p.x;
  const int nchunk = K / 8;
  float xv[NCH][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int ch = tid + c * kDenseWarps * 32;
    if (ch < nchunk) {
      const float4 lo = reinterpret_cast<const float4*>(x)[2 * ch];
      const float4 hi = reinterpret_cast<const float4*>(x)[2 * ch + 1];
      xv[c][0] = lo.x; xv[c][1] = lo.y; xv[c][2] = lo.z; xv[c][3] = lo.w;
      xv[c][4] = hi.x; xv[c][5] = hi.y; xv[c][6] = hi.z; xv[c][7] = hi.w;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) xv[c][j] = 0.f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(xv[c][j], xv[c][j], ss);
  }
  if (a.p.norm_w) {
    ss = warp_sum(ss);
    if (lane == 0) ssq[warp] = ss;
    named_sync(1, kDenseWarps * 32);
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kDenseWarps; ++w) tot += ssq[w];
    const float r = 1.0f / sqrtf(tot / (float)K + a.p.rms_eps);
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int ch = tid + c * kDenseWarps * 32;
      if (ch < nchunk) {
        const float4 lo = reinterpret_cast<const float4*>(a.p.norm_w)[2 * ch];
        const float4 hi = reinterpret_cast<const float4*>(a.p.norm_w)[2 * ch + 1];
        const float wn[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) xv[c][j] = __fmul_rn(__fmul_rn(xv[c][j], r), wn[j]);  // (x * r) * w
      }
    }
  }
  // biases and residuals of this CTA's rows, staged once (one load latency instead of one per tile)
  if (a.pre) {
    for (int i = tid; i < r_end - r_begin; i += kDenseWarps * 32) {
      const int row = r_begin + i;
      int s = 0;
      while (s + 1 < a.p.n_seg && row >= a.seg_start[s + 1]) ++s;
      const ns_dense_seg_t& sg = a.p.seg[s];
      const int lr = row - a.seg_start[s];
      pre_b[i] = sg.bias ? sg.bias[lr] : 0.f;
      pre_r[i] = sg.residual ? sg.residual[lr] : 0.f;
    }
    named_sync(1, kDenseWarps * 32);
  }
  griddep_launch_dependents();

  int done = 0;  // tiles consumed
  bool failed = false;
  for (int i = 0; i < n_tiles; ++i) {
    const int slot = i % nst;
    // a wait that runs out marks this thread; the tile's barrier below ORs the marks, so every
    // compute thread leaves the loop at the same tile (the stage's bytes are then not used)
    const bool landed = mbar_wait_bounded(&full[slot], (uint32_t)((i / nst) & 1));
    const uint8_t* st = stages + (size_t)slot * a.stage_bytes;
    float acc[kDenseTileRows];
#pragma unroll
    for (int r = 0; r < kDenseTileRows; ++r) acc[r] = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int ch = tid + c * kDenseWarps * 32;
      if (ch < nchunk) {
#pragma unroll
        for (int r = 0; r < kDenseTileRows; ++r) {
          if (r >= tr) break;
          const uint4 w = *reinterpret_cast<const uint4*>(st + (size_t)r * row_bytes + (size_t)ch * 16);
          const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            acc[r] = fmaf(__uint_as_float(ww[j] << 16), xv[c][2 * j], acc[r]);
            acc[r] = fmaf(__uint_as_float(ww[j] & 0xFFFF0000u), xv[c][2 * j + 1], acc[r]);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);  // this warp is done reading the stage
    const float v = reduce8_rows(acc, lane);
    float* rb = red + (i & 1) * kDenseWarps * kDenseTileRows;
    if ((lane & 3) == 0) rb[warp * kDenseTileRows + dense_row_of(lane)] = v;
    if (named_sync_or(1, kDenseWarps * 32, !landed)) {
      failed = true;
      break;
    }
    done = i + 1;
    if (tid < tr) {
      const int row = r_begin + i * tr + tid;
      if (row < r_end) {
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < kDenseWarps; ++w) sum += rb[w * kDenseTileRows + tid];
        int s = 0;
        while (s + 1 < a.p.n_seg && row >= a.seg_start[s + 1]) ++s;
        const ns_dense_seg_t& sg = a.p.seg[s];
        const int lr = row - a.seg_start[s];
        float y;
        if (a.pre) {
          const int i = row - r_begin;
          y = sg.bias ? sum + pre_b[i] : sum;
          if (sg.residual) y = pre_r[i] + y;
        } else {
          y = sg.bias ? sum + sg.bias[lr] : sum;
          if (sg.residual) y = sg.residual[lr] + y;
        }
        sg.y[lr] = y;
      }
    }
  }
  if (failed && tid == 0) {
    // let the copies still in flight land before the CTA's shared memory goes away: wait (bounded)
    // for the producer to stop, then for every tile it issued and nobody consumed
    raise_device_error(NS_DEVERR_COPY_WAIT);
    const uint64_t t0 = globaltimer_ns();
    while (!s_prod_done && globaltimer_ns() - t0 < 2 * kWaitLimitNs) __nanosleep(256);
    if (s_prod_done)
      for (int j = done; j < s_issued; ++j) (void)mbar_wait_bounded(&full[j % nst], (uint32_t)((j / nst) & 1));
  }
}

template <int NCH>
static int launch_dense(const DenseArgs& a, int grid, size_t smem, cudaStream_t s) {
  auto kern = dense_gemv_kernel<NCH>;
  // the kernel's whole budget, not this launch's size: one function serves launches of several sizes,
  // and a captured graph replays each of them against the attribute's value at replay time
  NS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)std::max(smem, (size_t)kDenseSmemBudget)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kDenseThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  NS_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a));
  return NS_OK;
}

}  // namespace ns

extern "C" int ns_dense_gemv(const ns_dense_gemv_t* p, ns_stream_t stream) {
  using namespace ns;
  if (!p) return fail(NS_ERR_INVALID, "ns_dense_gemv: null parameters");
  if (p->w_dtype != NS_BF16) return fail(NS_ERR_UNSUPPORTED, "ns_dense_gemv: weights must be bf16 (NS_BF16)");
  if (p->K < 8 || p->K % 8 || p->K > 8 * 256 * 4)
    return fail(NS_ERR_INVALID, "ns_dense_gemv: K=%d must be a multiple of 8 in 8..8192", p->K);
  if (p->n_seg < 1 || p->n_seg > NS_DENSE_MAX_SEG)
    return fail(NS_ERR_INVALID, "ns_dense_gemv: n_seg=%d outside 1..%d", p->n_seg, NS_DENSE_MAX_SEG);
  if (!p->x) return fail(NS_ERR_INVALID, "ns_dense_gemv: null x");
  for (int i = 0; i < NS_L2_PREFETCH_RANGES; ++i)
    if (p->l2.bytes[i] && (reinterpret_cast<uintptr_t>(p->l2.ptr[i]) & 15))
      return fail(NS_ERR_INVALID, "ns_dense_gemv: L2 prefetch range %d not 16-byte aligned", i);
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  if (!al16(p->x) || (p->norm_w && !al16(p->norm_w)))
    return fail(NS_ERR_INVALID, "ns_dense_gemv: x and norm_w must be 16-byte aligned");
  DenseArgs a;
  memset(&a, 0, sizeof a);
  a.p = *p;
  int total = 0;
  for (int s = 0; s < p->n_seg; ++s) {
    const ns_dense_seg_t& sg = p->seg[s];
    if (!sg.w || !sg.y || sg.rows < 1) return fail(NS_ERR_INVALID, "ns_dense_gemv: segment %d: null pointer or no rows", s);
    if (!al16(sg.w)) return fail(NS_ERR_INVALID, "ns_dense_gemv: segment %d weights not 16-byte aligned", s);
    a.seg_start[s] = total;
    total += sg.rows;
  }
  a.seg_start[p->n_seg] = total;
  a.total_rows = total;
  int nsm = 0;
  int st = num_sms(&nsm);
  if (st) return st;
  bool any_extra = false;
  for (int s = 0; s < p->n_seg; ++s) any_extra |= p->seg[s].bias != nullptr || p->seg[s].residual != nullptr;
  const size_t fixed = 2 * kDenseMaxStages * 8 + (2 * kDenseWarps * kDenseTileRows + kDenseWarps) * 4 +
                       (size_t)2 * kDensePreRows * 4 + 128;
  a.tile_rows = kDenseTileRows;
  while (a.tile_rows > 1 && (size_t)3 * a.tile_rows * p->K * 2 > kDenseSmemBudget - fixed) a.tile_rows /= 2;
  const int grid = std::max(1, std::min(nsm, (total + a.tile_rows - 1) / a.tile_rows));
  a.stage_bytes = a.tile_rows * p->K * 2;
  a.pre = any_extra && (total + grid - 1) / grid <= kDensePreRows;
  a.stages = (int)std::min<size_t>(kDenseMaxStages, (kDenseSmemBudget - fixed) / a.stage_bytes);
  if (a.stages < 2) return fail(NS_ERR_UNSUPPORTED, "ns_dense_gemv: K=%d leaves fewer than 2 stages", p->K);
  const size_t smem = (size_t)a.stages * a.stage_bytes + fixed;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int nch = (p->K / 8 + kDenseWarps * 32 - 1) / (kDenseWarps * 32);
  switch (nch) {
    case 1: return launch_dense<1>(a, grid, smem, s);
    case 2: return launch_dense<2>(a, grid, smem, s);
    case 3: return launch_dense<3>(a, grid, smem, s);
    default: return launch_dense<4>(a, grid, smem, s);
  }
}
