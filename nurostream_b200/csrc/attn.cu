// ns_attn_decode: one decode token of GPT-OSS attention over an HBM-resident KV cache.
//
// Stands in for the core of GptOssModel._attention_block (neurostream/model/gpt_oss.py:101-114):
// apply_rope on q and the new k (neurostream/compute/ops.py:141-151, the YaRN tables of
// gpt_oss.py:44-58 supplied by the caller), KVCache.append (neurostream/model/qwen3.py:74-85),
// repeat_kv (ops.py:154-159) and sink_attention (gpt_oss.py:73-87): causal softmax over the visible
// keys plus one learned sink logit per query head, with the sliding window on the layers that use it.
// The q/k/v projections before it and the output projection after it are ns_dense_gemv launches.
//
// Work split (flash-decoding): one CTA per (kv head g, key split s).  The CTA's 8 warps are the 8
// query heads that share kv head g (GQA); within a 64-key block lane j scores keys j and j + 32
// against its head's rotated q held in registers, and accumulates p * V for dims 2j, 2j + 1.  Keys
// are walked in blocks of 64 with an online softmax (running max, sum and output), double-buffered
// in shared memory by cp.async.  The splits of kv head g are one thread-block cluster: each CTA leaves
// (max, sum, output) per head in its shared memory and the cluster's rank-0 CTA merges them, in split
// order and together with the sinks, through distributed shared memory (no global round trip, and a
// result that does not depend on CTA timing).
//
// The token's own key and value come from the projection output (rotated here); the CTA of the last
// split also writes them into the cache at slot pos for later tokens.  Under programmatic dependent
// launch the first two key blocks are requested before griddepcontrol.wait: cache slots below pos were
// written by kernels at least two launches back, which the stream's chain invariant (no kernel lets
// its dependents launch before its own wait) has already completed.  Slot pos itself is never read
// from the cache in this launch.

namespace ns {

constexpr int kAttnHd = 64;             // head_dim this kernel is built for
constexpr int kAttnBlock = 64;          // keys per block
constexpr int kAttnKPitch = 68;         // floats per K row in shared memory: 16-byte loads stay conflict-free
constexpr int kAttnMaxRep = 8;          // query heads per kv head (warps per CTA)
constexpr int kAttnThreads = kAttnMaxRep * 32;
constexpr int kAttnMaxSplits = 16;      // key splits of one kv head = CTAs of one cluster

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Barrier over every thread of every CTA of the cluster, ordering shared-memory writes before it
// against reads after it (a launch without clusters is a cluster of one CTA).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory variable in the CTA of cluster rank r.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, int r) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(addr), "r"(r));
  return out;
}
__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

struct AttnArgs {
  ns_attn_decode_t p;
  int splits;         // key splits per kv head (the cluster size)
};

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// x * cos + rotate_half(x) * sin, for element d of a 64-wide head (two roundings and a sum, as
// the reference's fp32 expression evaluates it).
__device__ __forceinline__ float rope_at(const float* x, const float* c, const float* s, int d) {
  const float rot = d < kAttnHd / 2 ? -x[d + kAttnHd / 2] : x[d - kAttnHd / 2];
  return __fadd_rn(__fmul_rn(x[d], c[d]), __fmul_rn(rot, s[d]));
}

struct AttnSmem {
  float sk[2][kAttnBlock][kAttnKPitch];  // key blocks (double buffer)
  float sv[2][kAttnBlock][kAttnHd];      // value blocks
  float sq[kAttnMaxRep][kAttnHd];        // rotated q of the group's heads
  float snew[2][kAttnHd];                // rotated new key, new value
  float sp[kAttnMaxRep][kAttnBlock];     // probabilities of the current block
  float pm[kAttnMaxRep], pl[kAttnMaxRep];  // this split's running max and sum per head
  float pacc[kAttnMaxRep][kAttnHd];        // and its unnormalised output
};

__global__ void __launch_bounds__(kAttnThreads, 1) attn_decode_kernel(AttnArgs a) {
  const ns_attn_decode_t& p = a.p;
  extern __shared__ __align__(128) uint8_t attn_smem[];
  AttnSmem& S = *reinterpret_cast<AttnSmem*>(attn_smem);
  auto& sk = S.sk;
  auto& sv = S.sv;
  auto& sq = S.sq;
  auto& snew = S.snew;
  auto& sp = S.sp;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = blockIdx.x / a.splits, s = blockIdx.x % a.splits;
  const int n_rep = p.n_head / p.n_head_kv;
  const int64_t cache_base = (int64_t)g * p.max_ctx * kAttnHd;

  const int pos = *p.pos;  // written before this step's kernels (see the chain invariant above)
  if (pos < 0 || pos >= p.max_ctx) {  // a position outside the cache: flag it, touch nothing
    if (tid == 0 && blockIdx.x == 0) raise_device_error(NS_DEVERR_ROUTE);
    griddep_wait();
    griddep_launch_dependents();
    return;
  }
  const int k_lo = p.window > 0 ? max(0, pos - p.window + 1) : 0;
  const int n_keys = pos - k_lo + 1;
  const int j0 = k_lo + (int)((int64_t)n_keys * s / a.splits);
  const int j1 = k_lo + (int)((int64_t)n_keys * (s + 1) / a.splits);
  const int n_blocks = (j1 - j0 + kAttnBlock - 1) / kAttnBlock;

  // request key block b (cache slots below pos only; slot pos comes from the projection)
  auto load_block = [&](int b) {
    const int kb = j0 + b * kAttnBlock, nb = min(kAttnBlock, j1 - kb);
    float(*dk)[kAttnKPitch] = sk[b & 1];
    float(*dv)[kAttnHd] = sv[b & 1];
    for (int i = tid; i < nb * (kAttnHd / 4); i += kAttnThreads) {
      const int r = i / (kAttnHd / 4), c = (i % (kAttnHd / 4)) * 4;
      if (kb + r == pos) continue;
      const int64_t off = cache_base + (int64_t)(kb + r) * kAttnHd + c;
      cp_async16(&dk[r][c], p.k_cache + off);
      cp_async16(&dv[r][c], p.v_cache + off);
    }
    cp_async_commit();
  };
  // both buffers' blocks before the wait: with 2,048 keys over 16 splits that is all of them
  if (n_blocks > 0) load_block(0);
  if (n_blocks > 1) load_block(1);
  if (tid == 0) l2_prefetch_share(p.l2, blockIdx.x, gridDim.x);  // the next kernels' weights (hint)

  griddep_wait();
  // rotated q of this group's heads, the new key (rotated) and value
  const float* cs = p.rope_cos + (int64_t)pos * kAttnHd;
  const float* sn = p.rope_sin + (int64_t)pos * kAttnHd;
  const float* q = p.qkv + (int64_t)g * n_rep * kAttnHd;
  const float* kn = p.qkv + (int64_t)p.n_head * kAttnHd + (int64_t)g * kAttnHd;
  const float* vn = p.qkv + (int64_t)(p.n_head + p.n_head_kv) * kAttnHd + (int64_t)g * kAttnHd;
  for (int i = tid; i < n_rep * kAttnHd; i += kAttnThreads) {
    const int h = i / kAttnHd, d = i % kAttnHd;
    sq[h][d] = rope_at(q + h * kAttnHd, cs, sn, d);
  }
  if (tid < kAttnHd) {
    snew[0][tid] = rope_at(kn, cs, sn, tid);
    snew[1][tid] = vn[tid];
  }
  __syncthreads();
  griddep_launch_dependents();
  if (s == a.splits - 1 && tid < kAttnHd) {  // append the token's key and value to the cache
    p.k_cache[cache_base + (int64_t)pos * kAttnHd + tid] = snew[0][tid];
    p.v_cache[cache_base + (int64_t)pos * kAttnHd + tid] = snew[1][tid];
  }

  const bool head_ok = warp < n_rep;
  float qr[kAttnHd];
#pragma unroll
  for (int d = 0; d < kAttnHd; ++d) qr[d] = head_ok ? sq[warp][d] : 0.f;
  float m = -INFINITY, l = 0.f, acc0 = 0.f, acc1 = 0.f;

  for (int b = 0; b < n_blocks; ++b) {
    // block b has landed once at most the one after it is still in flight
    if (b + 1 < n_blocks)
      cp_async_wait<1>();
    else
      cp_async_wait<0>();
    const int kb = j0 + b * kAttnBlock, nb = min(kAttnBlock, j1 - kb);
    float(*dk)[kAttnKPitch] = sk[b & 1];
    float(*dv)[kAttnHd] = sv[b & 1];
    if (pos >= kb && pos < kb + nb && tid < kAttnHd) {
      dk[pos - kb][tid] = snew[0][tid];
      dv[pos - kb][tid] = snew[1][tid];
    }
    __syncthreads();
    if (head_ok) {
      float sc[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int j = lane + 32 * u;
        float dot = 0.f;
        if (j < nb) {
#pragma unroll
          for (int c = 0; c < kAttnHd / 4; ++c) {
            const float4 kv = *reinterpret_cast<const float4*>(&dk[j][4 * c]);
            dot = fmaf(qr[4 * c], kv.x, dot);
            dot = fmaf(qr[4 * c + 1], kv.y, dot);
            dot = fmaf(qr[4 * c + 2], kv.z, dot);
            dot = fmaf(qr[4 * c + 3], kv.w, dot);
          }
          sc[u] = dot * p.scale;
        } else {
          sc[u] = -INFINITY;
        }
      }
      float bm = fmaxf(sc[0], sc[1]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, o));
      const float m_new = fmaxf(m, bm);
      const float corr = expf(m - m_new);  // 0 on the first block (m = -inf)
      const float p0 = expf(sc[0] - m_new), p1 = expf(sc[1] - m_new);
      sp[warp][lane] = p0;
      sp[warp][lane + 32] = p1;
      l = l * corr + warp_sum(p0 + p1);
      acc0 *= corr;
      acc1 *= corr;
      m = m_new;
      __syncwarp();
      for (int j = 0; j < nb; ++j) {
        const float pj = sp[warp][j];
        const float2 vv = *reinterpret_cast<const float2*>(&dv[j][2 * lane]);
        acc0 = fmaf(pj, vv.x, acc0);
        acc1 = fmaf(pj, vv.y, acc1);
      }
    }
    __syncthreads();  // the buffer of block b is free for block b + 2
    if (b + 2 < n_blocks) load_block(b + 2);
  }

  // this split's partial result per head, in shared memory; the splits of kv head g form one thread
  // block cluster, and its rank-0 CTA merges them through distributed shared memory
  if (head_ok) {
    if (lane == 0) {
      S.pm[warp] = m;
      S.pl[warp] = l;
    }
    S.pacc[warp][2 * lane] = acc0;
    S.pacc[warp][2 * lane + 1] = acc1;
  }
  cluster_sync_all();
  if (cluster_rank() == 0 && head_ok) {
    // merge in split order, with each head's sink as one more logit
    const int h = g * n_rep + warp;
    const uint32_t pm = smem_addr(&S.pm[warp]), pl = smem_addr(&S.pl[warp]);
    const uint32_t pa = smem_addr(&S.pacc[warp][2 * lane]);
    float ms[kAttnMaxSplits], ls[kAttnMaxSplits], a0[kAttnMaxSplits], a1[kAttnMaxSplits];
#pragma unroll
    for (int t = 0; t < kAttnMaxSplits; ++t)
      if (t < a.splits) {  // all remote loads first
        ms[t] = ld_cluster_f32(mapa_shared(pm, t));
        ls[t] = ld_cluster_f32(mapa_shared(pl, t));
        a0[t] = ld_cluster_f32(mapa_shared(pa, t));
        a1[t] = ld_cluster_f32(mapa_shared(pa + 4, t));
      }
    float mt = p.sinks ? p.sinks[h] : -INFINITY;
#pragma unroll
    for (int t = 0; t < kAttnMaxSplits; ++t)
      if (t < a.splits) mt = fmaxf(mt, ms[t]);
    float lt = p.sinks ? expf(p.sinks[h] - mt) : 0.f, o0 = 0.f, o1 = 0.f;
#pragma unroll
    for (int t = 0; t < kAttnMaxSplits; ++t)
      if (t < a.splits && ms[t] != -INFINITY) {  // a split with no keys adds nothing
        const float f = expf(ms[t] - mt);
        lt = fmaf(ls[t], f, lt);
        o0 = fmaf(a0[t], f, o0);
        o1 = fmaf(a1[t], f, o1);
      }
    p.out[(int64_t)h * kAttnHd + 2 * lane] = o0 / lt;
    p.out[(int64_t)h * kAttnHd + 2 * lane + 1] = o1 / lt;
  }
  cluster_sync_all();  // every CTA's shared memory stays alive until rank 0 has read it
}

static int g_attn_max_cluster = 0;  // largest cluster the device schedules for this kernel (8 or 16)

static int attn_max_cluster() {
  if (g_attn_max_cluster) return g_attn_max_cluster;
  int best = 8;
  if (cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess &&
      cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(AttnSmem)) ==
          cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kAttnMaxSplits);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = sizeof(AttnSmem);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kAttnMaxSplits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, attn_decode_kernel, &cfg) == cudaSuccess && n >= 1) best = kAttnMaxSplits;
  }
  (void)cudaGetLastError();
  g_attn_max_cluster = best;
  return best;
}

static int attn_plan(const ns_attn_decode_t* p, int* splits) {
  if (!p) return fail(NS_ERR_INVALID, "ns_attn_decode: null parameters");
  if (p->head_dim != kAttnHd) return fail(NS_ERR_UNSUPPORTED, "ns_attn_decode: head_dim %d (only 64)", p->head_dim);
  if (p->n_head_kv < 1 || p->n_head < p->n_head_kv || p->n_head % p->n_head_kv ||
      p->n_head / p->n_head_kv > kAttnMaxRep)
    return fail(NS_ERR_UNSUPPORTED, "ns_attn_decode: %d query heads over %d kv heads (at most %d per kv head)",
                p->n_head, p->n_head_kv, kAttnMaxRep);
  if (p->max_ctx < 1 || p->window < 0) return fail(NS_ERR_INVALID, "ns_attn_decode: bad max_ctx / window");
  // keys per split <= one 64-key block where the cluster size allows it
  const int keys = p->window > 0 ? std::min(p->window + 1, p->max_ctx) : p->max_ctx;
  *splits = std::max(1, std::min(attn_max_cluster(), (keys + kAttnBlock - 1) / kAttnBlock));
  return NS_OK;
}

}  // namespace ns

extern "C" int ns_attn_workspace_bytes(const ns_attn_decode_t* p, size_t* bytes) {
  using namespace ns;
  if (!bytes) return fail(NS_ERR_INVALID, "ns_attn_workspace_bytes: null output");
  int splits = 0;
  int st = attn_plan(p, &splits);
  if (st) return st;
  *bytes = 0;  // the splits merge through distributed shared memory
  return NS_OK;
}

extern "C" int ns_attn_decode(const ns_attn_decode_t* p, void* workspace, size_t workspace_bytes, ns_stream_t stream) {
  using namespace ns;
  (void)workspace;
  (void)workspace_bytes;
  int splits = 0;
  int st = attn_plan(p, &splits);
  if (st) return st;
  if (!p->pos || !p->qkv || !p->rope_cos || !p->rope_sin || !p->k_cache || !p->v_cache || !p->out)
    return fail(NS_ERR_INVALID, "ns_attn_decode: null pointer");
  if ((reinterpret_cast<uintptr_t>(p->k_cache) | reinterpret_cast<uintptr_t>(p->v_cache)) & 15)
    return fail(NS_ERR_INVALID, "ns_attn_decode: caches must be 16-byte aligned");
  for (int i = 0; i < NS_L2_PREFETCH_RANGES; ++i)
    if (p->l2.bytes[i] && (reinterpret_cast<uintptr_t>(p->l2.ptr[i]) & 15))
      return fail(NS_ERR_INVALID, "ns_attn_decode: L2 prefetch range %d not 16-byte aligned", i);
  AttnArgs a;
  a.p = *p;
  a.splits = splits;
  NS_CUDA_TRY(cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)sizeof(AttnSmem)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p->n_head_kv * splits);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = sizeof(AttnSmem);
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = splits;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  NS_CUDA_TRY(cudaLaunchKernelEx(&cfg, attn_decode_kernel, a));
  return NS_OK;
}

// ------------------------------------------------------------------------------------------------
// ns_embed: the token's embedding row widened to fp32 (Qwen3Model.embed, qwen3.py:266-275:
// `self.w('token_embd.weight')[tokens]`), with the token id read from device memory so that one
// captured graph serves every token.

namespace ns {

__global__ void embed_kernel(const void* table, int dtype, int64_t rows, int H, const int32_t* token, float* out) {
  griddep_wait();
  const int t = *token;
  griddep_launch_dependents();
  if (t < 0 || t >= rows) {
    if (blockIdx.x == 0 && threadIdx.x == 0) raise_device_error(NS_DEVERR_ROUTE);
    return;
  }
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < H; i += gridDim.x * blockDim.x)
    out[i] = load_float(table, dtype, (int64_t)t * H + i);
}

}  // namespace ns

extern "C" int ns_embed(const void* table, int dtype, int64_t rows, int H, const int32_t* token, float* out,
                        ns_stream_t stream) {
  using namespace ns;
  if (!table || !token || !out || rows < 1 || H < 1) return fail(NS_ERR_INVALID, "ns_embed: bad arguments");
  if (!float_type_ok(dtype)) return fail(NS_ERR_INVALID, "ns_embed: bad dtype %d", dtype);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((H + 255) / 256);
  cfg.blockDim = dim3(256);
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  NS_CUDA_TRY(cudaLaunchKernelEx(&cfg, embed_kernel, table, dtype, rows, H, token, out));
  return NS_OK;
}
