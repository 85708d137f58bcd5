// MoE prefill: the experts of T tokens as a grouped GEMM on the tcgen05 tensor cores.
//
// Replaces the prefill walk of the reference (neurostream/compute/blockffn.py:171-176, 220-229;
// neurostream/moe/router.py:158-166): per routed expert, dequantize each block of its stacked
// rows and multiply the expert's tokens by it, one expert after another.  Here every expert's
// weights stream from HBM once for all of its tokens (and once more per extra group of 16):
//
//   pf_norm_kernel     RMSNorm of the T tokens
//   pf_logits_kernel   router logits (tiled product)
//   pf_topk_kernel     top-k and routing weights
//   pf_bucket_kernel   (token, expert) pairs sorted by (expert, token); groups of <= 32 pairs of one
//                      expert; the work items of both GEMM phases (pf_bucket_bits_kernel for T <= 2048)
//   pf_planes_kernel   digit planes of the normalised input, one copy per pair (pair order)
//   pf_gemm_kernel<0>  gate/up rows x planes of the group's tokens; clamped SwiGLU / SiLU*up in the
//                      epilogue, which writes the activation's digit planes (pair order)
//   pf_gemm_kernel<1>  down rows x activation planes -> one H-row of expert output per pair
//   pf_combine_kernel  out[t] = x[t] + sum over t's experts (ascending id) of w * y
//
// Arithmetic is the decode tensor-core kernel's (moe_tc.cu): weights are the A operand (128 rows of
// one expert, MXFP4 blocks moved into TMEM as they are, E8M0 bytes as UE8M0 block scales);
// activations are the B operand as 8 balanced radix-8 digit planes per token (an exact 24-bit
// fixed-point split per 32-element block), so a group of 32 tokens is N = 256.  D accumulates in
// fp32 in TMEM.  One kind::mxf4 MMA (M = 128, K = 64) takes the same time on B200 for any N up to
// 256, so the kernel makes N as large as the expert's tokens allow: groups of up to 32 tokens.
//
// GEMM kernel.  Persistent, one CTA per SM; items (expert, tile, group) are dealt round robin.  An
// expert's items are tile-major, so the groups of one tile (same weight bytes) run at the same time
// on neighbouring CTAs and a second read of the tile is served by L2.  A gate/up tile is 64
// neurons: its 128 M-rows are the 64 gate rows and the 64 up rows of those neurons, so both
// projections of a neuron land in one accumulator and the activation is formed in the epilogue; a
// down tile is 128 rows.  Per K chunk of 10 blocks: the producer issues the weight boxes (TMA row
// phases of 8-row groups), one 3-D TMA box of the group's planes (32 pairs x 10 blocks x 128
// bytes, which is the K-major operand layout as stored) and one bulk copy of the group's scale
// atoms; 12 repack warps move the weight blocks into TMEM; one thread issues the MMAs; 4 epilogue
// warps drain D.  Every wait is bounded; a wait that runs out raises a device error bit, stops the
// CTA's pipeline, lets in-flight copies and MMAs land, frees TMEM and returns.

namespace ns {

constexpr int kPfMaxTokens = 65536;
constexpr int kPfGroup = 32;                               // pairs per group: N = 8 planes x 32
constexpr int kPfChunk = 10;                               // K blocks (32 elements) per chunk
constexpr int kPfBoxW = 208;                               // TMA box row (bytes): >= 10*17 + 15; rows of a
                                                           // box land 52 words (20 banks) apart
constexpr int kPfBoxBytes = kPfBoxW * 16;                  // one row phase of 16 row groups (128 rows)
constexpr int kPfRawBytes = 8 * kPfBoxBytes;               // 8 row phases
constexpr int kPfRawStages = 3;                            // weight stages (staged GGUF rows)
constexpr int kPfBStages = 2;                              // activation-plane stages
constexpr int kPfSfbGroups = 3;                            // 4-block scale groups a 10-block chunk spans
constexpr int kPfBBytes = kPfGroup * kPfChunk * 128;       // planes of one chunk
constexpr int kPfBStageBytes = kPfBBytes + kPfSfbGroups * 1024;
// Weight operand of one chunk in shared memory: core matrices of 8 M-rows x 16 bytes (one block's
// payload), (M-row group g, block b) at g*1280 + b*128.
constexpr int kPfAOpBytes = 128 * kPfChunk * 16;
constexpr int kPfAStageBytes = kPfAOpBytes;
constexpr int kPfXchgBytes = kPfGroup * 128 * 4;
// TMEM columns: D [0, 256); weight scales 2 x 16 [256, 288) (3 atoms x 4 used); activation scales
// 2 x 24 [288, 336) (3 groups x 8: for N = 256 the scale of B row n sits in lane n % 32, column
// n / 32 of its group).
constexpr int kPfTmemSfa = 256, kPfTmemSfb = 288, kPfTmemCols = 512;
constexpr int kPfSmemBudget = 225 * 1024;
constexpr int kPfBucketSmem = 160 * 1024;                  // ids staged by the bucket kernel

struct PfHeader {
  int npairs, ngroups, nitems1, nitems2;
};

// Workspace pointers shared by the launches of one call.
struct PfWork {
  PfHeader* hdr;
  float* h;             // T x H normalised input
  int32_t* ids;         // T x k
  float* wts;           // T x k
  int32_t* tok_pair;    // T x k: pair index of (token, rank), -1 if the expert is not local
  int32_t* pair_tok;    // P
  float* pair_w;        // P
  int32_t* pair_gs;     // P: group << 5 | slot in group
  int4* grp;            // Gmax: local expert, first pair, pairs, 0
  int2* items1;         // phase-1 items: group, 64-neuron tile
  int2* items2;         // phase-2 items: group, 128-row tile
  uint8_t* planes1;     // P x nb_h x 128
  uint8_t* sf1;         // Gmax x sf1_bytes
  uint8_t* planes2;     // P x nb_f x 128
  uint8_t* sf2;         // Gmax x sf2_bytes
  float* ypair;         // P x H
  int sf1_bytes, sf2_bytes;
};

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* tmap, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
      ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
      : "memory");
}

// Byte of a group's scale image holding plane `pl` of slot `slot`, block `blk`: the image is one
// 1024-byte entry per 4 blocks, two 512-byte atoms (B rows 0..127, 128..255) as tcgen05.cp copies
// them; row m = 8*slot + pl of the B operand sits at 16*(m%32) + 4*((m/32)%4) + blk%4 of atom m/128.
__device__ __forceinline__ int pf_sf_off(int slot, int pl, int blk) {
  const int m = 8 * slot + pl;
  return (blk >> 2) * 1024 + (m >> 7) * 512 + 16 * (m & 31) + 4 * ((m >> 5) & 3) + (blk & 3);
}

// ----------------------------------------------------------------------------- routing

// RMSNorm of one token per CTA: h = x * rsqrt(mean(x^2) + eps) * norm_w (neurostream/model/
// gpt_oss.py:123-126 via the model's rms_norm), written to the workspace.
__global__ void __launch_bounds__(256) pf_norm_kernel(const ns_moe_layer_t p, PfWork w) {
  const int H = p.H, t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ float red[8];
  const float* x = p.x + (int64_t)t * H;
  float ss = 0.f;
  for (int i = tid; i < H; i += 256) ss = fmaf(x[i], x[i], ss);
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float r = p.norm_w ? 1.0f / sqrtf(tot / (float)H + p.rms_eps) : 1.0f;
  for (int i = tid; i < H; i += 256)
    w.h[(int64_t)t * H + i] = p.norm_w ? __fmul_rn(__fmul_rn(x[i], r), p.norm_w[i]) : x[i];
}

// Router logits L[t][e] = h[t] . W[e] + b[e] as a tiled product: a CTA of 128 threads owns 16
// tokens x 32 experts (2 x 2 per thread), K in steps of 64 through a 4-stage cp.async ring in
// shared memory (three steps in flight while one is multiplied); each output is one fp32 fma chain
// in ascending k.  WT: the router weight's element type (float, __half or __nv_bfloat16).
constexpr int kPfLgT = 16, kPfLgE = 32, kPfLgK = 64, kPfLgStages = 4;
constexpr int kPfLgHRow = kPfLgK * 4 + 16;                 // bytes per staged h row (padded)
constexpr int kPfLgWRow = kPfLgK * 4 + 16;                 // room for a staged W row of any type
constexpr int kPfLgStage = kPfLgT * kPfLgHRow + kPfLgE * kPfLgWRow;
template <typename WT>
__device__ __forceinline__ float pf_wval(const uint8_t* row, int k) {
  if constexpr (sizeof(WT) == 4) return reinterpret_cast<const float*>(row)[k];
  else if constexpr (std::is_same<WT, __half>::value) return __half2float(reinterpret_cast<const __half*>(row)[k]);
  else return __uint_as_float((uint32_t)reinterpret_cast<const unsigned short*>(row)[k] << 16);
}
template <typename WT>
__global__ void __launch_bounds__(128) pf_logits_kernel(const ns_moe_layer_t p, PfWork w, float* logits) {
  extern __shared__ __align__(16) uint8_t lg_sm[];
  const int H = p.H, E = p.n_expert, T = p.T;
  const int t0 = blockIdx.x * kPfLgT, e0 = blockIdx.y * kPfLgE;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;  // experts e0 + tx, +16; tokens t0 + ty, +8
  constexpr int kWBytes = kPfLgK * (int)sizeof(WT);            // bytes of one W row per step
  const int nsteps = H / kPfLgK;                                // H is a multiple of 64
  const WT* wbase = static_cast<const WT*>(p.router_w);
  auto issue = [&](int step) {
    if (step < nsteps) {
      uint8_t* st = lg_sm + (step % kPfLgStages) * kPfLgStage;
      const int k0 = step * kPfLgK;
      for (int i = tid; i < kPfLgT * (kPfLgK * 4 / 16); i += 128) {  // 16 chunks of 16 B per h row
        const int r = i >> 4, c = i & 15;
        const int t = min(t0 + r, T - 1);                                // rows past T: any valid row
        cp_async16(st + r * kPfLgHRow + 16 * c, w.h + (int64_t)t * H + k0 + 4 * c);
      }
      constexpr int kWChunks = kWBytes / 16;
      for (int i = tid; i < kPfLgE * kWChunks; i += 128) {
        const int r = i / kWChunks, c = i - r * kWChunks;
        const int e = min(e0 + r, E - 1);
        cp_async16(st + kPfLgT * kPfLgHRow + r * kPfLgWRow + 16 * c,
                   reinterpret_cast<const uint8_t*>(wbase + (int64_t)e * H + k0) + 16 * c);
      }
    }
    cp_async_commit();  // one group per step, empty ones included, so the wait counts stay uniform
  };
  float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
  for (int s = 0; s < kPfLgStages - 1; ++s) issue(s);
  for (int step = 0; step < nsteps; ++step) {
    cp_async_wait<kPfLgStages - 2>();
    __syncthreads();  // the step's tiles are in; every thread is done with the slot reused below
    issue(step + kPfLgStages - 1);
    const uint8_t* st = lg_sm + (step % kPfLgStages) * kPfLgStage;
    const float* h0r = reinterpret_cast<const float*>(st + ty * kPfLgHRow);
    const float* h1r = reinterpret_cast<const float*>(st + (ty + 8) * kPfLgHRow);
    const uint8_t* w0r = st + kPfLgT * kPfLgHRow + tx * kPfLgWRow;
    const uint8_t* w1r = w0r + 16 * kPfLgWRow;
#pragma unroll 16
    for (int kk = 0; kk < kPfLgK; ++kk) {
      const float h0 = h0r[kk], h1 = h1r[kk], wv0 = pf_wval<WT>(w0r, kk), wv1 = pf_wval<WT>(w1r, kk);
      acc[0][0] = fmaf(h0, wv0, acc[0][0]);
      acc[0][1] = fmaf(h0, wv1, acc[0][1]);
      acc[1][0] = fmaf(h1, wv0, acc[1][0]);
      acc[1][1] = fmaf(h1, wv1, acc[1][1]);
    }
  }
  cp_async_wait<0>();
#pragma unroll
  for (int a = 0; a < 2; ++a)
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      const int t = t0 + ty + 8 * a, e = e0 + tx + 16 * b;
      if (t < T && e < E) logits[(int64_t)t * E + e] = acc[a][b] + (p.router_b ? p.router_b[e] : 0.f);
    }
}

// Top-k and routing weights, one warp per token: neurostream/model/gpt_oss.py:116-121 (top-k of the
// logits, softmax over the k) or neurostream/moe/router.py:59-69 (softmax, top-k, renormalise).
__global__ void __launch_bounds__(256) pf_topk_kernel(const ns_moe_layer_t p, PfWork w, const float* logits) {
  __shared__ int sid[8][NS_MAX_TOPK];
  __shared__ float swt[8][NS_MAX_TOPK];
  __shared__ float scr[8][NS_MAX_EXPERTS];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, k = p.k, E = p.n_expert;
  const int t = blockIdx.x * 8 + warp;
  if (t >= p.T) return;
  warp_route(logits + (int64_t)t * E, E, k, p.route_mode, sid[warp], swt[warp], scr[warp], lane);
  if (lane < k) {
    const int64_t o = (int64_t)t * k + lane;
    w.ids[o] = sid[warp][lane];
    w.wts[o] = swt[warp][lane];
    if (p.ids) p.ids[o] = sid[warp][lane];
    if (p.weights) p.weights[o] = swt[warp][lane];
  }
}

// ----------------------------------------------------------------------------- bucketing

// One CTA of 1024 threads.  Pairs of local expert e are the tokens routed to it in ascending
// order; experts ascend; e's pairs split into ceil(n/32) groups of near-equal size.
__global__ void __launch_bounds__(1024) pf_bucket_kernel(const ns_moe_layer_t p, PfWork w, int ns1, int nr2,
                                                        int ids_in_smem) {
  extern __shared__ int pf_ids_s[];  // T x k ids when they fit (ids_in_smem), else unused
  __shared__ int cnt[NS_MAX_EXPERTS], poff[NS_MAX_EXPERTS], goff[NS_MAX_EXPERTS];
  const int T = p.T, k = p.k, lo = p.expert_lo, nl = p.expert_hi - p.expert_lo;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int* ids = w.ids;
  if (ids_in_smem) {
    for (int i = tid; i < T * k; i += 1024) pf_ids_s[i] = w.ids[i];
    __syncthreads();
    ids = pf_ids_s;
  }
  for (int el = warp; el < nl; el += 32) {
    const int e = lo + el;
    int c = 0;
    for (int t0 = 0; t0 < T; t0 += 32) {
      const int t = t0 + lane;
      bool hit = false;
      if (t < T)
        for (int j = 0; j < k; ++j) hit |= ids[t * k + j] == e;
      c += __popc(__ballot_sync(0xffffffffu, hit));
    }
    if (lane == 0) cnt[el] = c;
  }
  for (int i = tid; i < T * k; i += 1024) w.tok_pair[i] = -1;
  __syncthreads();
  if (tid == 0) {
    int P = 0, G = 0;
    for (int el = 0; el < nl; ++el) {
      poff[el] = P;
      goff[el] = G;
      P += cnt[el];
      G += (cnt[el] + kPfGroup - 1) / kPfGroup;
    }
    w.hdr->npairs = P;
    w.hdr->ngroups = G;
    w.hdr->nitems1 = G * ns1;
    w.hdr->nitems2 = G * nr2;
  }
  __syncthreads();
  for (int el = warp; el < nl; el += 32) {
    const int e = lo + el, base = poff[el];
    int run = 0;
    for (int t0 = 0; t0 < T; t0 += 32) {
      const int t = t0 + lane;
      int jj = -1;
      if (t < T)
        for (int j = 0; j < k; ++j)
          if (ids[t * k + j] == e) jj = j;
      const unsigned m = __ballot_sync(0xffffffffu, jj >= 0);
      if (jj >= 0) {
        const int pos = base + run + __popc(m & ((1u << lane) - 1u));
        w.pair_tok[pos] = t;
        w.pair_w[pos] = w.wts[(int64_t)t * k + jj];
        w.tok_pair[(int64_t)t * k + jj] = pos;
      }
      run += __popc(m);
    }
    const int c = cnt[el], ng = (c + kPfGroup - 1) / kPfGroup, g0 = goff[el];
    for (int gi = lane; gi < ng; gi += 32) {
      const int bs = c / ng, rem = c - bs * ng;
      const int start = gi * bs + min(gi, rem), n = bs + (gi < rem ? 1 : 0);
      w.grp[g0 + gi] = make_int4(el, base + start, n, 0);
      for (int s = 0; s < n; ++s) w.pair_gs[base + start + s] = ((g0 + gi) << 5) | s;
    }
    for (int i = lane; i < ns1 * ng; i += 32) w.items1[ns1 * g0 + i] = make_int2(g0 + i % ng, i / ng);
    for (int i = lane; i < nr2 * ng; i += 32) w.items2[nr2 * g0 + i] = make_int2(g0 + i % ng, i / ng);
  }
}

// The same bucketing for T <= 2048 without serial loops: each local expert's tokens as a bitmap in
// shared memory (one atomicOr per routed pair), per-word prefix counts, then every pair finds its
// position (count of the expert's earlier tokens) in one step.  Same output as pf_bucket_kernel.
constexpr int kPfBitsMaxT = 2048;
__global__ void __launch_bounds__(1024) pf_bucket_bits_kernel(const ns_moe_layer_t p, PfWork w, int ns1, int nr2) {
  extern __shared__ uint32_t pf_bits[];  // nl x nw token bitmaps, then nl x nw 16-bit prefixes
  __shared__ int cnt[NS_MAX_EXPERTS], poff[NS_MAX_EXPERTS], goff[NS_MAX_EXPERTS];
  const int T = p.T, k = p.k, lo = p.expert_lo, nl = p.expert_hi - p.expert_lo, nw = (T + 31) / 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  unsigned short* pre = reinterpret_cast<unsigned short*>(pf_bits + nl * nw);
  for (int i = tid; i < nl * nw; i += 1024) pf_bits[i] = 0u;
  __syncthreads();
  for (int i = tid; i < T * k; i += 1024) {
    const int el = w.ids[i] - lo, t = i / k;
    if (el >= 0 && el < nl) atomicOr(&pf_bits[el * nw + (t >> 5)], 1u << (t & 31));
  }
  __syncthreads();
  for (int el = warp; el < nl; el += 32) {  // exclusive prefix of the word counts, per expert
    int running = 0;
    for (int w0 = 0; w0 < nw; w0 += 32) {
      const int wi = w0 + lane;
      const int c = wi < nw ? __popc(pf_bits[el * nw + wi]) : 0;
      int incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      if (wi < nw) pre[el * nw + wi] = (unsigned short)(running + incl - c);
      running += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) cnt[el] = running;
  }
  __syncthreads();
  if (tid == 0) {
    int P = 0, G = 0;
    for (int el = 0; el < nl; ++el) {
      poff[el] = P;
      goff[el] = G;
      P += cnt[el];
      G += (cnt[el] + kPfGroup - 1) / kPfGroup;
    }
    w.hdr->npairs = P;
    w.hdr->ngroups = G;
    w.hdr->nitems1 = G * ns1;
    w.hdr->nitems2 = G * nr2;
  }
  __syncthreads();
  for (int i = tid; i < T * k; i += 1024) {
    const int el = w.ids[i] - lo, t = i / k;
    if (el < 0 || el >= nl) {
      w.tok_pair[i] = -1;
      continue;
    }
    const int wd = el * nw + (t >> 5);
    const int r = pre[wd] + __popc(pf_bits[wd] & ((1u << (t & 31)) - 1u));  // earlier tokens of el
    const int pos = poff[el] + r;
    w.pair_tok[pos] = t;
    w.pair_w[pos] = w.wts[i];
    w.tok_pair[i] = pos;
    const int c = cnt[el], ng = (c + kPfGroup - 1) / kPfGroup, bs = c / ng, rem = c - bs * ng;
    int gi, sl;
    if (r < rem * (bs + 1)) {
      gi = r / (bs + 1);
      sl = r - gi * (bs + 1);
    } else {
      const int r2 = r - rem * (bs + 1);
      gi = rem + r2 / bs;
      sl = r2 - (gi - rem) * bs;
    }
    w.pair_gs[pos] = ((goff[el] + gi) << 5) | sl;
  }
  for (int el = warp; el < nl; el += 32) {
    const int c = cnt[el], ng = (c + kPfGroup - 1) / kPfGroup, g0 = goff[el], base = poff[el];
    for (int gi = lane; gi < ng; gi += 32) {
      const int bs = c / ng, rem = c - bs * ng;
      const int start = gi * bs + min(gi, rem), n = bs + (gi < rem ? 1 : 0);
      w.grp[g0 + gi] = make_int4(el, base + start, n, 0);
    }
    for (int i = lane; i < ns1 * ng; i += 32) w.items1[ns1 * g0 + i] = make_int2(g0 + i % ng, i / ng);
    for (int i = lane; i < nr2 * ng; i += 32) w.items2[nr2 * g0 + i] = make_int2(g0 + i % ng, i / ng);
  }
}

// ----------------------------------------------------------------------------- phase-1 planes

// Digit planes of h for every pair (pair order) and the group's scale atoms; one half-warp per
// (pair, block).
__global__ void __launch_bounds__(256) pf_planes_kernel(int H, PfWork w) {
  const int nb = H / 32;
  const int lane = threadIdx.x & 31, hl = lane & 15;
  const unsigned mask = 0xFFFFu << (lane & 16);
  const int hw0 = (blockIdx.x * blockDim.x + threadIdx.x) >> 4, nhw = (gridDim.x * blockDim.x) >> 4;
  const int units = w.hdr->npairs * nb;
  for (int u = hw0; u < units; u += nhw) {  // uniform per half-warp
    const int pr = u / nb, b = u - pr * nb;
    const int t = w.pair_tok[pr], gs = w.pair_gs[pr], g = gs >> 5, s = gs & 31;
    const float* hb = w.h + (int64_t)t * H + 32 * b + hl;
    halfwarp_block_planes(hb[0], hb[16], w.planes1 + ((size_t)pr * nb + b) * 128,
                          w.sf1 + (size_t)g * w.sf1_bytes + pf_sf_off(s, 0, b), 16, hl, mask);
  }
}

// ----------------------------------------------------------------------------- grouped GEMM

// Bounded wait (as tc_wait) that adds the time it spun to *acc (the tracer's per-role wait totals).
// Roles that wait for long stretches (producer, epilogue) sleep `nap` ns between polls, leaving the
// issue slots to the repack warps on the same sub-partitions.
template <int Nap = 0>
__device__ __forceinline__ bool pf_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                        unsigned long long* acc) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  const long long c0 = clock64();
  bool ok = true;
  while (!mbar_try_wait(bar, parity)) {
    if (*abort_flag) {
      ok = false;
      break;
    }
    if (Nap) __nanosleep(Nap);
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      raise_device_error(NS_DEVERR_COPY_WAIT);
      *abort_flag = 1;
      ok = false;
      break;
    }
  }
  *acc += (unsigned long long)(clock64() - c0);
  return ok;
}

// Tracer slots of the grouped GEMM (ns_moe_set_trace; per CTA, NS_TRACE_EVENTS values): start and
// end stamps (ns) and, per role, SM clock cycles spent waiting on each barrier.
enum { kPfEvStart = 0, kPfEvEnd, kPfEvProdEmptyRaw, kPfEvProdEmptyB, kPfEvProdItem, kPfEvRepFullRaw,
       kPfEvRepEmptyCan, kPfEvMmaFullCan, kPfEvMmaFullB, kPfEvMmaEmptyD, kPfEvEpiFullD, kPfEvEpiBusy,
       kPfEvMmaEnd, kPfEvProdEnd, kPfEvRepEnd, kPfEvEpiEnd };

struct PfGemmArgs {
  CUtensorMap tm_a[2];              // phase 0: gate rows, up rows (8-group boxes); phase 1: down rows
                                    // with 16-group boxes, and with 8-group boxes for a half tile
  CUtensorMap tm_b;                 // planes of this phase: (pairs, blocks, 128 bytes) as u32
  PfWork w;
  const float* bias0;               // phase 0 gate_b, phase 1 down_b (local experts x rows), or NULL
  const float* bias1;               // phase 0 up_b, or NULL
  int H, F, nb, rb, rows_e;         // rows_e: neurons (phase 0) or down rows (phase 1) per expert
  int act_mode;
  float alpha, limit;
  int off_raw, off_aop, off_b, off_xchg, off_bars, off_shared;
  unsigned long long* trace;        // per-CTA tracer slots, or NULL
};

struct PfShared {
  uint32_t tmem_base;
  int abort_flag;
};

// Rows of an item's tile: phase 0 a 64-neuron tile is 64 gate + 64 up rows (16 row groups); phase 1
// a tile is 128 down rows, or 64 for the last tile when H is an odd multiple of 64.
template <int PH>
__device__ __forceinline__ int pf_groups(int rows_e, int tile) {
  return PH == 0 ? 16 : (rows_e - 128 * tile >= 128 ? 16 : 8);
}

template <int PH>
__global__ void __launch_bounds__(kTcThreads, 1) pf_gemm_kernel(const __grid_constant__ PfGemmArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, c = blockIdx.x;
  const PfWork& W = a.w;
  const int2* items = PH == 0 ? W.items1 : W.items2;
  const uint8_t* sfimg = PH == 0 ? W.sf1 : W.sf2;
  const int sf_bytes = PH == 0 ? W.sf1_bytes : W.sf2_bytes;
  const int nb = a.nb, rb = a.rb, nq = (nb + kPfChunk - 1) / kPfChunk;
  constexpr int kTileStep = PH == 0 ? 64 : 128;  // expert rows (neurons or down rows) per tile

  uint8_t* raw = smem + a.off_raw;
  uint8_t* aop = smem + a.off_aop;
  uint8_t* bbuf = smem + a.off_b;
  float* xchg = reinterpret_cast<float*>(smem + a.off_xchg);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + a.off_bars);
  uint64_t* full_raw = bars;
  uint64_t* empty_raw = full_raw + kPfRawStages;
  uint64_t* full_b = empty_raw + kPfRawStages;
  uint64_t* empty_b = full_b + kPfBStages;
  uint64_t* full_can = empty_b + kPfBStages;
  uint64_t* empty_can = full_can + kTcCanStages;
  uint64_t* full_d = empty_can + kTcCanStages;
  uint64_t* empty_d = full_d + 1;
  uint64_t* mma_done = empty_d + 1;
  PfShared& S = *reinterpret_cast<PfShared*>(smem + a.off_shared);
  volatile int* abort_flag = &S.abort_flag;

  unsigned long long* tr = a.trace ? a.trace + (size_t)blockIdx.x * NS_TRACE_EVENTS : nullptr;
  unsigned long long w0 = 0, w1 = 0, w2 = 0;  // this thread's wait totals (role-specific)
  if (tid == 0 && tr) tr[kPfEvStart] = globaltimer_ns();
  if (tid == 0) {
    for (int s = 0; s < kPfRawStages; ++s) {
      mbar_init(&full_raw[s], 1);
      mbar_init(&empty_raw[s], kTcRepackWarps);
    }
    for (int s = 0; s < kPfBStages; ++s) {
      mbar_init(&full_b[s], 1);
      mbar_init(&empty_b[s], 1);
    }
    for (int s = 0; s < kTcCanStages; ++s) {
      mbar_init(&full_can[s], kTcRepackWarps);
      mbar_init(&empty_can[s], 1);
    }
    mbar_init(full_d, 1);
    mbar_init(empty_d, 4);
    mbar_init(mma_done, 1);
    fence_mbar_init();
    S.abort_flag = (smem_addr(smem) & 1023u) != 0;
    if (S.abort_flag) raise_device_error(NS_DEVERR_COPY_WAIT);
    prefetch_tmap(&a.tm_a[0]);
    prefetch_tmap(&a.tm_b);
  }
  if (warp == kTcMmaWarp) tmem_alloc(&S.tmem_base, kPfTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = S.tmem_base;
  const int nitems = PH == 0 ? W.hdr->nitems1 : W.hdr->nitems2;

  if (warp == kTcProducerWarp) {
    // ================================================================= producers (TMA)
    // Lane 0 streams the weights, lane 1 the activation planes, each as far ahead as its own ring
    // allows: the weight prefetch depth does not wait for plane stages.
    if (lane == 0) {
      const uint64_t policy = l2_evict_first_policy();
      int n = 0;  // weight chunks issued
      for (int i = c; i < nitems && !*abort_flag; i += G) {
        const long long ti = tr ? clock64() : 0;
        const int2 it = items[i];
        const int4 g = W.grp[it.x];
        const int gv = pf_groups<PH>(a.rows_e, it.y);
        const int y0 = (g.x * a.rows_e + kTileStep * it.y) / 8;
        if (tr) w2 += (unsigned long long)(clock64() - ti);
        for (int q = 0; q < nq; ++q, ++n) {
          const int wb = kPfChunk * q;
          const int st = n % kPfRawStages;
          if (!pf_wait<64>(&empty_raw[st], ((n / kPfRawStages) & 1) ^ 1, abort_flag, &w0)) break;
          mbar_arrive_expect_tx(&full_raw[st], (uint32_t)(8 * gv * kPfBoxW));
          uint8_t* dst = raw + st * kPfRawBytes;
#pragma unroll 1
          for (int j = 0; j < 8; ++j) {
            const int x0 = ((j * rb + 17 * wb) & ~15) >> 1;  // u16 elements
            if (PH == 0) {  // gate rows to row groups 0..7, up rows to 8..15 of the row phase
              tma_load_2d_hint(dst + j * kPfBoxBytes, &a.tm_a[0], x0, y0, &full_raw[st], policy);
              tma_load_2d_hint(dst + j * kPfBoxBytes + 8 * kPfBoxW, &a.tm_a[1], x0, y0, &full_raw[st], policy);
            } else {
              tma_load_2d_hint(dst + j * kPfBoxBytes, gv == 16 ? &a.tm_a[0] : &a.tm_a[1], x0, y0, &full_raw[st],
                               policy);
            }
          }
        }
      }
      // let every issued load land before the CTA can exit
      for (int q = max(0, n - kPfRawStages); q < n; ++q)
        mbar_wait_bounded(&full_raw[q % kPfRawStages], (q / kPfRawStages) & 1);
      if (tr) {
        tr[kPfEvProdEmptyRaw] = w0;
        tr[kPfEvProdItem] = w2;
        tr[kPfEvProdEnd] = globaltimer_ns();
      }
    } else if (lane == 1) {
      int n = 0;  // plane chunks issued
      for (int i = c; i < nitems && !*abort_flag; i += G) {
        const int2 it = items[i];
        const int p0 = W.grp[it.x].y;
        for (int q = 0; q < nq; ++q, ++n) {
          const int wb = kPfChunk * q;
          const int bst = n % kPfBStages;
          if (!pf_wait<64>(&empty_b[bst], ((n / kPfBStages) & 1) ^ 1, abort_flag, &w1)) break;
          mbar_arrive_expect_tx(&full_b[bst], (uint32_t)kPfBStageBytes);
          uint8_t* bd = bbuf + bst * kPfBStageBytes;
          tma_load_3d(bd, &a.tm_b, 0, wb, p0, &full_b[bst]);  // 32 pairs (one box beats 8-pair boxes)
          bulk_g2s(bd + kPfBBytes, sfimg + (size_t)it.x * sf_bytes + (size_t)(wb >> 2) * 1024,
                   (uint32_t)(kPfSfbGroups * 1024), &full_b[bst]);
        }
      }
      for (int q = max(0, n - kPfBStages); q < n; ++q)
        mbar_wait_bounded(&full_b[q % kPfBStages], (q / kPfBStages) & 1);
      if (tr) tr[kPfEvProdEmptyB] = w1;
    }
  } else if (warp == kTcMmaWarp) {
    // ================================================================= MMA issuer
    if (lane == 0) {
      int n = 0, nit = 0;
      bool ok = true;
      for (int i = c; i < nitems && ok; i += G, ++nit) {
        const int2 it = items[i];
        const int ntok = W.grp[it.x].z;
        const int N = 16 * ((ntok + 1) / 2);
        if (!pf_wait<32>(empty_d, (nit & 1) ^ 1, abort_flag, &w2)) break;
        tc_fence_after();
        bool acc = false;
        for (int q = 0; q < nq; ++q, ++n) {
          const int wb = kPfChunk * q, nbc = min(kPfChunk, nb - wb);
          const int cst = n % kTcCanStages, bst = n % kPfBStages;
          if (!pf_wait<32>(&full_can[cst], (n / kTcCanStages) & 1, abort_flag, &w0) ||
              !pf_wait<32>(&full_b[bst], (n / kPfBStages) & 1, abort_flag, &w1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint8_t* bd = bbuf + bst * kPfBStageBytes;
          const uint32_t sfb_col = tbase + kPfTmemSfb + 24 * bst;
          // each copy costs tensor-pipe time: rows 128..255 of a group's scales only when N > 128
#pragma unroll
          for (int gq = 0; gq < kPfSfbGroups; ++gq)
#pragma unroll
            for (int h = 0; h < 2; ++h)
              if (h == 0 || N > 128)
                tc_cp_sf(sfb_col + 8 * gq + 4 * h, umma_desc(smem_addr(bd + kPfBBytes + 1024 * gq + 512 * h), 128, 128));
          const uint8_t* as = aop + cst * kPfAStageBytes;
          const uint32_t sfa_col = tbase + kPfTmemSfa + 16 * cst;  // stored by the repack warps
          // A: core matrix (M-row group g, block b) at g*1280 + b*128; B: (slot t, block b) at
          // t*1280 + b*128; both +256 bytes (+16) per MMA
          const uint64_t ad0 = umma_desc(smem_addr(as), 128, kPfChunk * 128);
          const uint64_t bd0 = umma_desc(smem_addr(bd), 128, kPfChunk * 128);
#pragma unroll
          for (int s = 0; s < kPfChunk / 2; ++s) {
            if (s < nbc / 2) {
              const uint32_t sfa_id = 2u * (s & 1);
              const int blk = wb + 2 * s;
              const uint32_t sfb_id = (uint32_t)(blk & 3);
              const uint32_t tsfa = (sfa_col + 4 * (s >> 1)) | (sfa_id << 30);
              const uint32_t tsfb = (sfb_col + 8 * ((blk >> 2) - (wb >> 2))) | (sfb_id << 30);
              mma_mxf4(tbase, ad0 + (uint64_t)(16 * s), bd0 + (uint64_t)(16 * s), idesc_mxf4(128, N, sfa_id, sfb_id),
                       tsfa, tsfb, acc ? 1u : 0u);
              acc = true;
            }
          }
          tc_commit(&empty_can[cst]);
          tc_commit(&empty_b[bst]);
        }
        if (!ok) break;
        tc_commit(full_d);
      }
      tc_commit(mma_done);
      mbar_wait_bounded(mma_done, 0);
      if (tr) {
        tr[kPfEvMmaFullCan] = w0;
        tr[kPfEvMmaFullB] = w1;
        tr[kPfEvMmaEmptyD] = w2;
        tr[kPfEvMmaEnd] = globaltimer_ns();
      }
    }
  } else if (tc_repack_index(warp) >= 0) {
    // ================================================================= repack warps
    // Each lane owns one staged row: tile row (Gr, j) = 8*Gr + j, read from row phase j, row group Gr
    // (quadrant q's three warps: Gr = 8*(q/2) + lane%8, j = 2*(lane/8) + q%2, so a warp's 32 reads
    // fall in distinct banks), and M-row m = 32*q + lane of the operand (tc_row_of(m) is its tile
    // row).  The three warps of a quadrant split a chunk's 10 blocks on scale-atom boundaries {0-3},
    // {4-7}, {8-9}.  Each block's 16 payload bytes go to the weight operand in shared memory (the 8
    // lanes of a 16-byte store phase write 8 distinct rows of one core matrix); the E8M0 bytes of a
    // 4-block atom form one TMEM word (lane m, column 4*atom + m/32), stored from registers so that
    // the tensor pipe spends no copy on them.
    const int rw = tc_repack_index(warp);
    const int q = rw / 3, wi = rw - 3 * q;
    const int Gr = 8 * (q >> 1) + (lane & 7), j = 2 * (lane >> 3) + (q & 1);
    const int m = 32 * q + lane;
    const uint32_t a_row = (uint32_t)((m >> 3) * (kPfChunk * 128) + (m & 7) * 16);
    const uint32_t taddr_lane = (uint32_t)(32 * q) << 16;
    const int nblk_w = wi < 2 ? 4 : 2;
    int n = 0;
    for (int i = c; i < nitems && !*abort_flag; i += G) {
      const int2 it = items[i];
      const bool row_ok = Gr < pf_groups<PH>(a.rows_e, it.y);
      for (int qc = 0; qc < nq && !*abort_flag; ++qc, ++n) {
        const int wb = kPfChunk * qc, nbc = min(kPfChunk, nb - wb);
        const int st = n % kPfRawStages, cst = n % kTcCanStages;
        if (!pf_wait(&full_raw[st], (n / kPfRawStages) & 1, abort_flag, &w0)) break;
        // this lane's row in the staged boxes, as a shared-window address (ld.shared below)
        const uint32_t rs = smem_addr(raw) + st * kPfRawBytes + j * kPfBoxBytes + Gr * kPfBoxW +
                            ((j * rb + 17 * wb) & 15);
        uint32_t wv[4][5];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int b = 4 * wi + u;
          const bool ok = row_ok && u < nblk_w && b < nbc;
          const uint32_t wa = (rs + 17 * b) & ~3u;
#pragma unroll
          for (int kk = 0; kk < 5; ++kk) wv[u][kk] = ok ? lds32(wa + 4 * kk) : 0u;
        }
        uint32_t pay[16], sw = 0u;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int b = 4 * wi + u;
          const uint32_t a0 = (rs + 17 * b) & 3u;  // the scale byte's offset in its word
          const uint32_t sh = 8 * ((a0 + 1) & 3);
          const bool whole = a0 == 3;                // payload is word-aligned: words 1..4
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            pay[4 * u + kk] = whole ? wv[u][kk + 1] : __funnelshift_r(wv[u][kk], wv[u][kk + 1], sh);
          sw |= ((wv[u][0] >> (8 * a0)) & 0xFFu) << (8 * u);
        }
        __syncwarp();  // every lane has consumed its staged words: the raw stage can be refilled
        if (lane == 0) mbar_arrive(&empty_raw[st]);
        // the operand stage must have been consumed by its earlier MMAs
        if (!pf_wait(&empty_can[cst], ((n / kTcCanStages) & 1) ^ 1, abort_flag, &w1)) break;
        const uint32_t as = smem_addr(aop) + cst * kPfAStageBytes;
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (u < nblk_w) sts128(as + a_row + (4 * wi + u) * 128, pay[4 * u], pay[4 * u + 1], pay[4 * u + 2], pay[4 * u + 3]);
        tc_fence_after();
        tmem_st_x1(tbase + kPfTmemSfa + 16 * cst + 4 * wi + q + taddr_lane, sw);
        fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_can[cst]);
      }
    }
    if (tr && rw == 0 && lane == 0) {
      tr[kPfEvRepFullRaw] = w0;
      tr[kPfEvRepEmptyCan] = w1;
      tr[kPfEvRepEnd] = globaltimer_ns();
    }
  } else if (tc_epi_quadrant(warp) >= 0) {
    // ================================================================= epilogue warps
    // D lane m is M-row m, tile row tc_row_of(m).  Phase 0: tile rows 0..63 are the gate rows and
    // 64..127 the up rows of the same 64 neurons; quadrants 0, 1 hold gate rows and quadrants 2, 3 the
    // up rows of the same neurons (lane for lane), which they hand over through shared memory.
    const int q = tc_epi_quadrant(warp);
    const int mrow = 32 * q + lane;
    const int row = tc_row_of(mrow);
    const bool is_up = PH == 0 && q >= 2;
    const int rl = PH == 0 ? (row & 63) : row;  // neuron (phase 0) or down row within the tile
    int nit = 0;
    for (int i = c; i < nitems; i += G, ++nit) {
      const int2 it = items[i];
      const int4 g = W.grp[it.x];
      const int ntok = g.z, p0 = g.y;
      const int r = kTileStep * it.y + rl;
      const bool valid = r < a.rows_e;
      float bias = 0.f;
      if (valid) {
        const float* bp = is_up ? a.bias1 : a.bias0;
        if (bp) bias = bp[(int64_t)g.x * a.rows_e + r];
      }
      if (!pf_wait<128>(full_d, nit & 1, abort_flag, &w0)) break;
      const long long tb = tr ? clock64() : 0;
      tc_fence_after();
      const uint32_t ta = tbase + ((uint32_t)(32 * q) << 16);
      float v[kPfGroup];
#pragma unroll
      for (int t4 = 0; t4 < kPfGroup; t4 += 4) {  // 4 tokens (32 columns) per round trip
        v[t4] = v[t4 + 1] = v[t4 + 2] = v[t4 + 3] = 0.f;
        if (t4 < ntok) {
          uint32_t x0[16], x1[16];
          tmem_ld_x16(ta + 8 * t4, x0);
          tmem_ld_x16(ta + 8 * t4 + 16, x1);
          tmem_wait_ld();
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            float s0 = 0.f, s1 = 0.f;
#pragma unroll
            for (int pl = 0; pl < 8; ++pl) {
              s0 += __uint_as_float(x0[8 * h2 + pl]);
              s1 += __uint_as_float(x1[8 * h2 + pl]);
            }
            v[t4 + h2] = s0;
            v[t4 + 2 + h2] = s1;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(empty_d);
      if (tr) w1 += (unsigned long long)(clock64() - tb);
      if (PH == 0) {
        if (is_up) {
#pragma unroll
          for (int t = 0; t < kPfGroup; ++t)
            if (t < ntok) xchg[t * 64 + rl] = v[t] + bias;
        }
        named_sync(1, 128);
        if (!is_up) {
#pragma unroll
          for (int t = 0; t < kPfGroup; ++t)
            if (t < ntok) xchg[t * 64 + rl] = activate(a.act_mode, v[t] + bias, xchg[t * 64 + rl], a.alpha, a.limit);
        }
        named_sync(1, 128);
        // digit planes of the tile's two 32-neuron blocks: warp q takes units (t, b) = u / 2, u % 2
        const int nb_f = a.F / 32;
        for (int u = q; u < 2 * ntok; u += 4) {
          const int t = u >> 1, b = u & 1, blk = 2 * it.y + b;
          const float av = xchg[t * 64 + 32 * b + lane];
          float m = fabsf(av);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
          const int be = block_be(m);
          const uint32_t cd = digit_planes(av, be);
          const uint32_t hi = __shfl_down_sync(0xffffffffu, cd, 16);
          const int pr = p0 + t;
          if (lane < 16) {
            uint8_t* img = W.planes2 + ((size_t)pr * nb_f + blk) * 128;
#pragma unroll
            for (int pl = 0; pl < 8; ++pl)
              img[pl * 16 + lane] = (uint8_t)(((cd >> (4 * pl)) & 15u) | (((hi >> (4 * pl)) & 15u) << 4));
          } else if (lane < 24) {
            const int pl = lane - 16;
            W.sf2[(size_t)it.x * W.sf2_bytes + pf_sf_off(t, pl, blk)] = (uint8_t)plane_scale(pl, be);
          }
        }
        named_sync(1, 128);
      } else {
#pragma unroll
        for (int t = 0; t < kPfGroup; ++t)
          if (t < ntok) xchg[t * 128 + row] = v[t] + bias;
        named_sync(1, 128);
        const int r0 = 128 * it.y;
        for (int t = q; t < ntok; t += 4)
          if (r0 + 4 * lane < a.rows_e)  // H - r0 is a multiple of 64
            __stcg(reinterpret_cast<float4*>(W.ypair + (size_t)(p0 + t) * a.H + r0) + lane,
                   *reinterpret_cast<const float4*>(xchg + t * 128 + 4 * lane));
        named_sync(1, 128);
      }
    }
    if (tr && q == 0 && lane == 0) {
      tr[kPfEvEpiFullD] = w0;
      tr[kPfEvEpiBusy] = w1;
      tr[kPfEvEpiEnd] = globaltimer_ns();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kTcMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tbase, kPfTmemCols);
  }
  if (tid == 0 && tr) tr[kPfEvEnd] = globaltimer_ns();
}

// ----------------------------------------------------------------------------- combine

// out[t] = x[t] + sum over t's local experts in ascending id of w * y (neurostream/model/gpt_oss.py:
// 139-173: out[rows] += w * expert(h[rows]) expert by expert, from zeros; then x + out).
__global__ void __launch_bounds__(256) pf_combine_kernel(const ns_moe_layer_t p, PfWork w) {
  const int H4 = p.H / 4, k = p.k;
  const int64_t n = (int64_t)p.T * H4;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < n; idx += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(idx / H4), r4 = (int)(idx - (int64_t)t * H4);
    int pe[NS_MAX_TOPK], pp[NS_MAX_TOPK];
    int m = 0;
    for (int j = 0; j < k; ++j) {
      const int pr = w.tok_pair[(int64_t)t * k + j];
      if (pr < 0) continue;
      const int e = w.ids[(int64_t)t * k + j];
      int i = m++;
      while (i > 0 && pe[i - 1] > e) {  // insertion by expert id
        pe[i] = pe[i - 1];
        pp[i] = pp[i - 1];
        --i;
      }
      pe[i] = e;
      pp[i] = pr;
    }
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i = 0; i < m; ++i) {
      const float wt = w.pair_w[pp[i]];
      const float4 y = __ldcg(reinterpret_cast<const float4*>(w.ypair + (size_t)pp[i] * p.H) + r4);
      o.x = __fadd_rn(o.x, __fmul_rn(wt, y.x));
      o.y = __fadd_rn(o.y, __fmul_rn(wt, y.y));
      o.z = __fadd_rn(o.z, __fmul_rn(wt, y.z));
      o.w = __fadd_rn(o.w, __fmul_rn(wt, y.w));
    }
    if (p.add_residual) {
      const float4 x = reinterpret_cast<const float4*>(p.x + (int64_t)t * p.H)[r4];
      o = make_float4(__fadd_rn(x.x, o.x), __fadd_rn(x.y, o.y), __fadd_rn(x.z, o.z), __fadd_rn(x.w, o.w));
    }
    reinterpret_cast<float4*>(p.out + (int64_t)t * p.H)[r4] = o;
  }
}

// ----------------------------------------------------------------------------- host side

struct PfPlan {
  int P, Gmax, ns1, nr2, nb_h, nb_f, sf1_bytes, sf2_bytes;
  size_t off_hdr, off_h, off_ids, off_wts, off_tok_pair, off_pair_tok, off_pair_w, off_pair_gs, off_grp, off_it1,
      off_it2, off_planes1, off_sf1, off_planes2, off_sf2, off_ypair, total;
};

static int pf_validate(const ns_moe_layer_t* p, PfPlan* pl) {
  if (!p) return fail(NS_ERR_INVALID, "ns_moe_prefill_grouped: null parameters");
  if (p->T < 1 || p->T > kPfMaxTokens)
    return fail(NS_ERR_INVALID, "ns_moe_prefill_grouped: T=%d outside 1..%d", p->T, kPfMaxTokens);
  if (p->n_expert < 1 || p->n_expert > NS_MAX_EXPERTS)
    return fail(NS_ERR_INVALID, "ns_moe_prefill_grouped: n_expert=%d outside 1..%d", p->n_expert, NS_MAX_EXPERTS);
  if (p->k < 1 || p->k > NS_MAX_TOPK || p->k > p->n_expert)
    return fail(NS_ERR_INVALID, "ns_moe_prefill_grouped: k=%d outside 1..min(%d, n_expert)", p->k, NS_MAX_TOPK);
  if (p->expert_lo < 0 || p->expert_hi > p->n_expert || p->expert_lo >= p->expert_hi)
    return fail(NS_ERR_INVALID, "ns_moe_prefill_grouped: bad local expert range [%d, %d)", p->expert_lo, p->expert_hi);
  if (p->route_mode != NS_ROUTE_TOPK_SOFTMAX && p->route_mode != NS_ROUTE_SOFTMAX_TOPK_NORM)
    return fail(NS_ERR_INVALID, "ns_moe_prefill_grouped: bad route mode %d", p->route_mode);
  if (p->act_mode != NS_ACT_CLAMPED_SWIGLU && p->act_mode != NS_ACT_SILU_MUL)
    return fail(NS_ERR_INVALID, "ns_moe_prefill_grouped: bad activation mode %d", p->act_mode);
  if (!float_type_ok(p->router_dtype))
    return fail(NS_ERR_INVALID, "ns_moe_prefill_grouped: bad router dtype %d", p->router_dtype);
  if (p->ggml_type != NS_GGML_MXFP4)
    return fail(NS_ERR_UNSUPPORTED, "ns_moe_prefill_grouped: expert type %d (the grouped GEMM takes MXFP4)",
                p->ggml_type);
  if (p->H <= 0 || p->F <= 0 || p->H % 64 || p->F % 64 || p->H > 8192 || p->F > 8192)
    return fail(NS_ERR_INVALID, "ns_moe_prefill_grouped: H=%d and F=%d must be multiples of 64 up to 8192", p->H,
                p->F);
  if (!p->x || !p->out || !p->router_w || !p->gate_w || !p->up_w || !p->down_w)
    return fail(NS_ERR_INVALID, "ns_moe_prefill_grouped: null tensor");
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  if (!al16(p->gate_w) || !al16(p->up_w) || !al16(p->down_w) || !al16(p->x) || !al16(p->out) || !al16(p->router_w))
    return fail(NS_ERR_INVALID, "ns_moe_prefill_grouped: expert tensors, router_w, x and out must be 16-byte aligned");
  const int64_t P = (int64_t)p->T * p->k;
  const int nl = p->expert_hi - p->expert_lo;
  pl->P = (int)P;
  pl->Gmax = (int)std::min<int64_t>(P, (P + kPfGroup - 1) / kPfGroup + nl);
  pl->ns1 = p->F / 64;  // gate/up tiles of 64 neurons
  pl->nr2 = (p->H + 127) / 128;
  pl->nb_h = p->H / 32;
  pl->nb_f = p->F / 32;
  pl->sf1_bytes = ((pl->nb_h + 3) / 4 + 2) * 1024;  // + the groups a last chunk's scale copy reads past
  pl->sf2_bytes = ((pl->nb_f + 3) / 4 + 2) * 1024;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 256);
    return o;
  };
  pl->off_hdr = take(sizeof(PfHeader));
  pl->off_h = take((size_t)p->T * p->H * 4);
  pl->off_ids = take((size_t)P * 4);
  pl->off_wts = take((size_t)P * 4);
  pl->off_tok_pair = take((size_t)P * 4);
  pl->off_pair_tok = take((size_t)P * 4);
  pl->off_pair_w = take((size_t)P * 4);
  pl->off_pair_gs = take((size_t)P * 4);
  pl->off_grp = take((size_t)pl->Gmax * 16);
  pl->off_it1 = take((size_t)pl->Gmax * pl->ns1 * 8);
  pl->off_it2 = take((size_t)pl->Gmax * pl->nr2 * 8);
  pl->off_planes1 = take((size_t)P * pl->nb_h * 128);
  pl->off_sf1 = take((size_t)pl->Gmax * pl->sf1_bytes);
  pl->off_planes2 = take((size_t)P * pl->nb_f * 128);
  pl->off_sf2 = take((size_t)pl->Gmax * pl->sf2_bytes);
  pl->off_ypair = take(std::max((size_t)P * p->H, (size_t)p->T * p->n_expert) * 4);  // + logits scratch
  pl->total = off;
  return NS_OK;
}

// Planes of `P` pairs x `nb` blocks x 128 bytes as a 3-D u32 tensor; box = 32 pairs x 10 blocks.
static int make_planes_map(CUtensorMap* m, const uint8_t* base, int P, int nb) {
  EncodeTiledFn fn;
  int st = get_encode_fn(&fn);
  if (st) return st;
  const cuuint64_t dims[3] = {32, (cuuint64_t)nb, (cuuint64_t)P};
  const cuuint64_t strides[2] = {128, (cuuint64_t)nb * 128};
  const cuuint32_t box[3] = {32, (cuuint32_t)kPfChunk, (cuuint32_t)kPfGroup};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<uint8_t*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NS_ERR_CUDA, "cuTensorMapEncodeTiled (planes) failed (%d)", (int)r);
  return NS_OK;
}

// Tensor map over `rows` GGUF rows of `rb` bytes viewed as (rows/8) groups of 8*rb bytes (16-bit
// elements); the box is kPfBoxW bytes of `box_groups` consecutive groups.
static int pf_row_group_map(CUtensorMap* m, const uint8_t* base, int64_t rows, int rb, int box_groups) {
  EncodeTiledFn fn;
  int st = get_encode_fn(&fn);
  if (st) return st;
  const cuuint64_t dims[2] = {(cuuint64_t)4 * rb, (cuuint64_t)(rows / 8)};  // u16 elements (rb is even)
  const cuuint64_t strides[1] = {(cuuint64_t)8 * rb};
  const cuuint32_t box[2] = {(cuuint32_t)(kPfBoxW / 2), (cuuint32_t)box_groups};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint8_t*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NS_ERR_CUDA, "cuTensorMapEncodeTiled (expert rows) failed (%d)", (int)r);
  return NS_OK;
}

static size_t pf_gemm_smem(PfGemmArgs* a) {
  size_t off = 0;
  a->off_raw = 0;
  off += (size_t)kPfRawStages * kPfRawBytes;
  a->off_aop = (int)off;
  off += (size_t)kTcCanStages * kPfAStageBytes;
  a->off_b = (int)off;
  off += (size_t)kPfBStages * kPfBStageBytes;
  off = align_up(off, 128);
  a->off_xchg = (int)off;
  off += kPfXchgBytes;
  a->off_bars = (int)off;
  off += 32 * 8;
  a->off_shared = (int)off;
  off += sizeof(PfShared);
  return align_up(off, 128);
}

template <int PH>
static int pf_launch_gemm(const PfGemmArgs& a, int grid, size_t smem, cudaStream_t s) {
  auto kern = pf_gemm_kernel<PH>;
  NS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)std::max(smem, (size_t)kPfSmemBudget)));
  kern<<<grid, kTcThreads, smem, s>>>(a);
  NS_CUDA_TRY(cudaGetLastError());
  return NS_OK;
}

static int pf_run(const ns_moe_layer_t* p, const PfPlan& pl, uint8_t* ws, cudaStream_t s) {
  int nsm = 0;
  int st = num_sms(&nsm);
  if (st) return st;
  PfWork w;
  memset(&w, 0, sizeof w);
  w.hdr = reinterpret_cast<PfHeader*>(ws + pl.off_hdr);
  w.h = reinterpret_cast<float*>(ws + pl.off_h);
  w.ids = reinterpret_cast<int32_t*>(ws + pl.off_ids);
  w.wts = reinterpret_cast<float*>(ws + pl.off_wts);
  w.tok_pair = reinterpret_cast<int32_t*>(ws + pl.off_tok_pair);
  w.pair_tok = reinterpret_cast<int32_t*>(ws + pl.off_pair_tok);
  w.pair_w = reinterpret_cast<float*>(ws + pl.off_pair_w);
  w.pair_gs = reinterpret_cast<int32_t*>(ws + pl.off_pair_gs);
  w.grp = reinterpret_cast<int4*>(ws + pl.off_grp);
  w.items1 = reinterpret_cast<int2*>(ws + pl.off_it1);
  w.items2 = reinterpret_cast<int2*>(ws + pl.off_it2);
  w.planes1 = ws + pl.off_planes1;
  w.sf1 = ws + pl.off_sf1;
  w.planes2 = ws + pl.off_planes2;
  w.sf2 = ws + pl.off_sf2;
  w.ypair = reinterpret_cast<float*>(ws + pl.off_ypair);
  w.sf1_bytes = pl.sf1_bytes;
  w.sf2_bytes = pl.sf2_bytes;

  // 1. route: RMSNorm, logits, top-k
  pf_norm_kernel<<<p->T, 256, 0, s>>>(*p, w);
  NS_CUDA_TRY(cudaGetLastError());
  float* logits = reinterpret_cast<float*>(w.ypair);  // scratch until phase 2 writes ypair
  {
    const dim3 lgrid((p->T + kPfLgT - 1) / kPfLgT, (p->n_expert + kPfLgE - 1) / kPfLgE);
    const size_t lsmem = (size_t)kPfLgStages * kPfLgStage;
    if (p->router_dtype == NS_F32) {
      NS_CUDA_TRY(cudaFuncSetAttribute(pf_logits_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lsmem));
      pf_logits_kernel<float><<<lgrid, 128, lsmem, s>>>(*p, w, logits);
    } else if (p->router_dtype == NS_F16) {
      NS_CUDA_TRY(cudaFuncSetAttribute(pf_logits_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lsmem));
      pf_logits_kernel<__half><<<lgrid, 128, lsmem, s>>>(*p, w, logits);
    } else {
      NS_CUDA_TRY(cudaFuncSetAttribute(pf_logits_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)lsmem));
      pf_logits_kernel<__nv_bfloat16><<<lgrid, 128, lsmem, s>>>(*p, w, logits);
    }
    NS_CUDA_TRY(cudaGetLastError());
  }
  pf_topk_kernel<<<(p->T + 7) / 8, 256, 0, s>>>(*p, w, logits);
  NS_CUDA_TRY(cudaGetLastError());
  // 2. bucket: token bitmaps for up to 2048 tokens, else the serial scan (ids staged in shared
  // memory when they fit)
  const int nl = p->expert_hi - p->expert_lo;
  const size_t bits_bytes = (size_t)nl * ((p->T + 31) / 32) * 6;
  if (p->T <= kPfBitsMaxT && bits_bytes <= (size_t)kPfBucketSmem) {
    NS_CUDA_TRY(cudaFuncSetAttribute(pf_bucket_bits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPfBucketSmem));
    pf_bucket_bits_kernel<<<1, 1024, align_up(bits_bytes, 16), s>>>(*p, w, pl.ns1, pl.nr2);
  } else {
    const size_t ids_bytes = (size_t)p->T * p->k * 4;
    const bool ids_smem = ids_bytes <= (size_t)kPfBucketSmem;
    NS_CUDA_TRY(cudaFuncSetAttribute(pf_bucket_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPfBucketSmem));
    pf_bucket_kernel<<<1, 1024, ids_smem ? ids_bytes : 0, s>>>(*p, w, pl.ns1, pl.nr2, ids_smem ? 1 : 0);
  }
  NS_CUDA_TRY(cudaGetLastError());
  // 3. phase-1 planes
  {
    const int64_t hw = (int64_t)pl.P * pl.nb_h;  // half-warps of work at most
    const int grid = (int)std::min<int64_t>((hw * 16 + 255) / 256, (int64_t)nsm * 8);
    pf_planes_kernel<<<std::max(grid, 1), 256, 0, s>>>(p->H, w);
    NS_CUDA_TRY(cudaGetLastError());
  }
  // 4. + 5. grouped GEMMs
  PfGemmArgs a;
  memset(&a, 0, sizeof a);
  a.w = w;
  a.H = p->H;
  a.F = p->F;
  a.act_mode = p->act_mode;
  a.alpha = p->alpha;
  a.limit = p->limit;
  a.trace = g_trace_buf[trace_slot()];
  unsigned long long* trace2 = a.trace;  // the down-projection launch: second half when the buffer has room
  if (a.trace && g_trace_bytes[trace_slot()] >= (size_t)2 * nsm * NS_TRACE_EVENTS * 8) trace2 += (size_t)nsm * NS_TRACE_EVENTS;
  const size_t smem = pf_gemm_smem(&a);
  if (smem > (size_t)kPfSmemBudget)
    return fail(NS_ERR_UNSUPPORTED, "ns_moe_prefill_grouped: layout needs %zu bytes of shared memory", smem);
  const int grid = nsm;
  const int rb_h = (int)row_bytes_of(p->ggml_type, p->H), rb_f = (int)row_bytes_of(p->ggml_type, p->F);
  {
    const int64_t rows = (int64_t)nl * p->F;
    st = pf_row_group_map(&a.tm_a[0], p->gate_w, rows, rb_h, 8);
    if (!st) st = pf_row_group_map(&a.tm_a[1], p->up_w, rows, rb_h, 8);
    if (!st) st = make_planes_map(&a.tm_b, w.planes1, pl.P, pl.nb_h);
    if (st) return st;
    a.nb = pl.nb_h;
    a.rb = rb_h;
    a.rows_e = p->F;
    a.bias0 = p->gate_b;
    a.bias1 = p->up_b;
    st = pf_launch_gemm<0>(a, grid, smem, s);
    if (st) return st;
  }
  {
    const int64_t rows = (int64_t)nl * p->H;
    st = pf_row_group_map(&a.tm_a[0], p->down_w, rows, rb_f, 16);
    if (!st) st = pf_row_group_map(&a.tm_a[1], p->down_w, rows, rb_f, 8);
    if (!st) st = make_planes_map(&a.tm_b, w.planes2, pl.P, pl.nb_f);
    if (st) return st;
    a.nb = pl.nb_f;
    a.rb = rb_f;
    a.rows_e = p->H;
    a.bias0 = p->down_b;
    a.bias1 = nullptr;
    a.trace = trace2;
    st = pf_launch_gemm<1>(a, grid, smem, s);
    if (st) return st;
  }
  // 6. combine
  {
    const int64_t n = (int64_t)p->T * (p->H / 4);
    const int cgrid = (int)std::min<int64_t>((n + 255) / 256, (int64_t)nsm * 16);
    pf_combine_kernel<<<cgrid, 256, 0, s>>>(*p, w);
    NS_CUDA_TRY(cudaGetLastError());
  }
  return NS_OK;
}

}  // namespace ns

extern "C" int ns_moe_prefill_workspace_bytes(const ns_moe_layer_t* p, size_t* bytes) {
  using namespace ns;
  if (!bytes) return fail(NS_ERR_INVALID, "ns_moe_prefill_workspace_bytes: null output");
  PfPlan pl;
  int st = pf_validate(p, &pl);
  if (st) return st;
  *bytes = pl.total;
  return NS_OK;
}

extern "C" int ns_moe_prefill_grouped(const ns_moe_layer_t* p, void* workspace, size_t workspace_bytes,
                                      ns_stream_t stream) {
  using namespace ns;
  PfPlan pl;
  int st = pf_validate(p, &pl);
  if (st) return st;
  if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return fail(NS_ERR_INVALID, "ns_moe_prefill_grouped: workspace must be 256-byte aligned");
  if (workspace_bytes < pl.total)
    return fail(NS_ERR_SIZE, "ns_moe_prefill_grouped: workspace %zu bytes < %zu needed", workspace_bytes, pl.total);
  return pf_run(p, pl, reinterpret_cast<uint8_t*>(workspace), reinterpret_cast<cudaStream_t>(stream));
}
