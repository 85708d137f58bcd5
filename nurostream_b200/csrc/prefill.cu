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
//   pf_bucket_kernel   (token, expert) pairs sorted by (expert, token); groups of <= 16 pairs of one
//                      expert; the work items of both GEMM phases
//   pf_planes_kernel   digit planes of the normalised input, one copy per pair (pair order)
//   pf_gemm_kernel<0>  gate/up rows x planes of the group's tokens; clamped SwiGLU / SiLU*up in the
//                      epilogue, which writes the activation's digit planes (pair order)
//   pf_gemm_kernel<1>  down rows x activation planes -> one H-row of expert output per pair
//   pf_combine_kernel  out[t] = x[t] + sum over t's experts (ascending id) of w * y
//
// Arithmetic is the decode tensor-core kernel's (moe_tc.cu): weights are the A operand (128 rows of
// one expert, MXFP4 blocks moved into TMEM as they are, E8M0 bytes as UE8M0 block scales);
// activations are the B operand as 8 balanced radix-8 digit planes per token (an exact 24-bit
// fixed-point split per 32-element block), so a group of 16 tokens is N = 128.  D accumulates in
// fp32 in TMEM.
//
// GEMM kernel.  Persistent, one CTA per SM; items (expert, 128-row tile, group) are dealt round
// robin.  An expert's items are tile-major, so the groups of one tile (same weight bytes) run at
// the same time on neighbouring CTAs and the second read of the tile is served by L2.  Per K chunk
// of 14 blocks: the producer issues the weight boxes (8 TMA boxes of row phases, as in the decode
// kernel), one 3-D TMA box of the group's planes (16 pairs x 14 blocks x 128 bytes, which is the
// K-major operand layout as stored) and one bulk copy of the group's scale atoms; 12 repack warps
// move the weight blocks into TMEM; one thread issues the MMAs; 4 epilogue warps drain D.
// Every wait is bounded; a wait that runs out raises a device error bit, stops the CTA's pipeline,
// lets in-flight copies and MMAs land, frees TMEM and returns.

namespace ns {

constexpr int kPfMaxTokens = 65536;
constexpr int kPfGroup = 16;                               // pairs per group: N = 8 planes x 16
constexpr int kPfRawStages = 4;                            // weight stages (kTcRawBytes each)
constexpr int kPfBStages = 2;                              // activation-plane stages
constexpr int kPfSfbAtoms = 5;                             // 4-block scale atoms a 14-block chunk spans
constexpr int kPfBBytes = kPfGroup * kTcChunk * 128;       // planes of one chunk
constexpr int kPfBStageBytes = kPfBBytes + kPfSfbAtoms * 512;
constexpr int kPfXchgBytes = kPfGroup * 128 * 4;
// TMEM columns: D gate [0, 128) and up [128, 256) (phase 2: [0, 128)); weights (A) 2 stages x 64
// [256, 384); weight scales 2 x 16 [384, 416); activation scales 2 x 20 [416, 456).
constexpr int kPfTmemUp = 128, kPfTmemA = 256, kPfTmemSfa = 384, kPfTmemSfb = 416, kPfTmemCols = 512;
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
  int32_t* pair_gs;     // P: group << 4 | slot in group
  int4* grp;            // Gmax: local expert, first pair, pairs, 0
  int2* items1;         // phase-1 items: group, 128-neuron tile
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

// Byte of scale atom `atom` holding plane `pl` of slot `slot`, block `blk` (blk % 4 within the
// atom): row m = 8*slot + pl of the B operand at 16*(m%32) + 4*(m/32) + blk%4.
__device__ __forceinline__ int pf_sf_byte(int slot, int pl, int blk) {
  return 16 * (8 * (slot & 3) + pl) + 4 * (slot >> 2) + (blk & 3);
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
// tokens x 32 experts (2 x 2 per thread), K in steps of 64 through shared memory, the next step's
// tiles loaded into registers while the current one is multiplied; each output is one fp32 fma
// chain in ascending k.
constexpr int kPfLgT = 16, kPfLgE = 32, kPfLgK = 64;
__global__ void __launch_bounds__(128) pf_logits_kernel(const ns_moe_layer_t p, PfWork w, float* logits) {
  __shared__ float hs[kPfLgT][kPfLgK + 1];
  __shared__ float ws[kPfLgE][kPfLgK + 1];
  const int H = p.H, E = p.n_expert, T = p.T;
  const int t0 = blockIdx.x * kPfLgT, e0 = blockIdx.y * kPfLgE;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;  // experts e0 + tx, +16; tokens t0 + ty, +8
  constexpr int kH = kPfLgT * kPfLgK / 128, kW = kPfLgE * kPfLgK / 128;  // loads per thread: 8, 16
  float hr[kH], wr[kW];
  auto load = [&](int k0) {
#pragma unroll
    for (int u = 0; u < kH; ++u) {
      const int i = tid + 128 * u, r = i / kPfLgK, c = i - r * kPfLgK;
      hr[u] = t0 + r < T ? w.h[(int64_t)(t0 + r) * H + k0 + c] : 0.f;
    }
    load_floats<kW>(p.router_w, p.router_dtype, [&](int u) -> int64_t {
      const int i = tid + 128 * u, r = i / kPfLgK, c = i - r * kPfLgK;
      return e0 + r < E ? (int64_t)(e0 + r) * H + k0 + c : -1;
    }, wr);
  };
  float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
  load(0);
  for (int k0 = 0; k0 < H; k0 += kPfLgK) {  // H is a multiple of 64
#pragma unroll
    for (int u = 0; u < kH; ++u) {
      const int i = tid + 128 * u;
      hs[i / kPfLgK][i % kPfLgK] = hr[u];
    }
#pragma unroll
    for (int u = 0; u < kW; ++u) {
      const int i = tid + 128 * u;
      ws[i / kPfLgK][i % kPfLgK] = wr[u];
    }
    __syncthreads();
    if (k0 + kPfLgK < H) load(k0 + kPfLgK);
#pragma unroll 16
    for (int kk = 0; kk < kPfLgK; ++kk) {
      const float h0 = hs[ty][kk], h1 = hs[ty + 8][kk], w0 = ws[tx][kk], w1 = ws[tx + 16][kk];
      acc[0][0] = fmaf(h0, w0, acc[0][0]);
      acc[0][1] = fmaf(h0, w1, acc[0][1]);
      acc[1][0] = fmaf(h1, w0, acc[1][0]);
      acc[1][1] = fmaf(h1, w1, acc[1][1]);
    }
    __syncthreads();
  }
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
// order; experts ascend; e's pairs split into ceil(n/16) groups of near-equal size.
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
      for (int s = 0; s < n; ++s) w.pair_gs[base + start + s] = ((g0 + gi) << 4) | s;
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
    const int t = w.pair_tok[pr], gs = w.pair_gs[pr], g = gs >> 4, s = gs & 15;
    const float* hb = w.h + (int64_t)t * H + 32 * b + hl;
    halfwarp_block_planes(hb[0], hb[16], w.planes1 + ((size_t)pr * nb + b) * 128,
                          w.sf1 + (size_t)g * w.sf1_bytes + (b >> 2) * 512 + pf_sf_byte(s, 0, b), 16, hl, mask);
  }
}

// ----------------------------------------------------------------------------- grouped GEMM

// tc_wait that adds the time it spun to *acc (the tracer's per-role wait totals).
__device__ __forceinline__ bool pf_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                        unsigned long long* acc) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  const bool ok = tc_wait(bar, parity, abort_flag);
  *acc += globaltimer_ns() - t0;
  return ok;
}

// Tracer slots of the grouped GEMM (ns_moe_set_trace; per CTA, NS_TRACE_EVENTS values): start and
// end stamps and, per role, nanoseconds spent waiting on each barrier.
enum { kPfEvStart = 0, kPfEvEnd, kPfEvProdEmptyRaw, kPfEvProdEmptyB, kPfEvProdItem, kPfEvRepFullRaw,
       kPfEvRepEmptyCan, kPfEvMmaFullCan, kPfEvMmaFullB, kPfEvMmaEmptyD, kPfEvEpiFullD, kPfEvEpiBusy,
       kPfEvMmaEnd, kPfEvProdEnd, kPfEvRepEnd, kPfEvEpiEnd };

struct PfGemmArgs {
  CUtensorMap tm_a16[2], tm_a8[2];  // phase 1: gate, up; phase 2: down (index 0)
  CUtensorMap tm_b;                 // planes of this phase: (pairs, blocks, 128 bytes) as u32
  PfWork w;
  const float* bias0;               // phase 1 gate_b, phase 2 down_b (local experts x rows), or NULL
  const float* bias1;               // phase 1 up_b, or NULL
  int H, F, nb, rb, rows_e;         // rows_e: weight rows per expert (F or H)
  int act_mode;
  float alpha, limit;
  int off_raw, off_b, off_xchg, off_bars, off_shared;
  unsigned long long* trace;        // per-CTA tracer slots, or NULL
};

struct PfShared {
  uint32_t tmem_base;
  int abort_flag;
};

template <int PH>
__global__ void __launch_bounds__(kTcThreads, 1) pf_gemm_kernel(const __grid_constant__ PfGemmArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, c = blockIdx.x;
  constexpr int NH = PH == 0 ? 2 : 1;  // K halves of an item: gate then up, or down
  const PfWork& W = a.w;
  const int2* items = PH == 0 ? W.items1 : W.items2;
  const uint8_t* sfimg = PH == 0 ? W.sf1 : W.sf2;
  const int sf_bytes = PH == 0 ? W.sf1_bytes : W.sf2_bytes;
  const int nb = a.nb, rb = a.rb, nq = (nb + kTcChunk - 1) / kTcChunk;

  uint8_t* raw = smem + a.off_raw;
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
    prefetch_tmap(&a.tm_a16[0]);
    prefetch_tmap(&a.tm_b);
  }
  if (warp == kTcMmaWarp) tmem_alloc(&S.tmem_base, kPfTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = S.tmem_base;
  const int nitems = PH == 0 ? W.hdr->nitems1 : W.hdr->nitems2;

  if (warp == kTcProducerWarp) {
    // ================================================================= producer (TMA)
    if (lane == 0) {
      const uint64_t policy = l2_evict_first_policy();
      int n = 0, nbq = 0;  // weight chunks and plane stages issued
      for (int i = c; i < nitems && !*abort_flag; i += G) {
        const uint64_t ti = tr ? globaltimer_ns() : 0;
        const int2 it = items[i];
        const int4 g = W.grp[it.x];
        const int rows = min(128, a.rows_e - 128 * it.y);
        const int gv = rows >= 128 ? 16 : rows / 8;
        const int y0 = (g.x * a.rows_e + 128 * it.y) / 8;
        if (tr) w2 += globaltimer_ns() - ti;
        // chunk order: (q, gate), (q, up), (q+1, gate), ..: the two halves of a K chunk share one
        // B stage (the planes of the same 14 blocks of h)
        for (int q = 0; q < nq && !*abort_flag; ++q) {
          const int wb = kTcChunk * q;
          for (int hf = 0; hf < NH; ++hf, ++n) {
            const CUtensorMap* tm = gv == 16 ? &a.tm_a16[hf] : &a.tm_a8[hf];
            const int st = n % kPfRawStages, bst = nbq % kPfBStages;
            // both waits before any copy of this step is issued (an abort then leaves none unaccounted)
            if (!pf_wait(&empty_raw[st], ((n / kPfRawStages) & 1) ^ 1, abort_flag, &w0)) break;
            if (hf == 0 && !pf_wait(&empty_b[bst], ((nbq / kPfBStages) & 1) ^ 1, abort_flag, &w1)) break;
            mbar_arrive_expect_tx(&full_raw[st], (uint32_t)(8 * gv * kTcBoxW));
            uint8_t* dst = raw + st * kTcRawBytes;
#pragma unroll 1
            for (int j = 0; j < 8; ++j) {
              const int x0 = ((j * rb + 17 * wb) & ~15) >> 1;  // u16 elements
              tma_load_2d_hint(dst + j * kTcBoxBytes, tm, x0, y0, &full_raw[st], policy);
            }
            if (hf == 0) {
              mbar_arrive_expect_tx(&full_b[bst], (uint32_t)kPfBStageBytes);
              uint8_t* bd = bbuf + bst * kPfBStageBytes;
              tma_load_3d(bd, &a.tm_b, 0, wb, g.y, &full_b[bst]);
              bulk_g2s(bd + kPfBBytes, sfimg + (size_t)it.x * sf_bytes + (size_t)(wb >> 2) * 512,
                       (uint32_t)(kPfSfbAtoms * 512), &full_b[bst]);
              ++nbq;
            }
          }
        }
      }
      // let every issued load land before the CTA can exit
      for (int q = max(0, n - kPfRawStages); q < n; ++q)
        mbar_wait_bounded(&full_raw[q % kPfRawStages], (q / kPfRawStages) & 1);
      for (int q = max(0, nbq - kPfBStages); q < nbq; ++q)
        mbar_wait_bounded(&full_b[q % kPfBStages], (q / kPfBStages) & 1);
      if (tr) {
        tr[kPfEvProdEmptyRaw] = w0;
        tr[kPfEvProdEmptyB] = w1;
        tr[kPfEvProdItem] = w2;
        tr[kPfEvProdEnd] = globaltimer_ns();
      }
    }
  } else if (warp == kTcMmaWarp) {
    // ================================================================= MMA issuer
    if (lane == 0) {
      int n = 0, nit = 0, nbq = 0;
      bool ok = true;
      for (int i = c; i < nitems && ok; i += G, ++nit) {
        const int2 it = items[i];
        const int ntok = W.grp[it.x].z;
        const int N = 16 * ((ntok + 1) / 2);
        if (!pf_wait(empty_d, (nit & 1) ^ 1, abort_flag, &w2)) break;
        tc_fence_after();
        bool acc_h[2] = {false, false};  // gate / up accumulators written in this item
        for (int q = 0; q < nq && ok; ++q) {
          const int wb = kTcChunk * q, nbc = min(kTcChunk, nb - wb);
          const int bst = nbq % kPfBStages;
          if (!pf_wait(&full_b[bst], (nbq / kPfBStages) & 1, abort_flag, &w1)) {
            ok = false;
            break;
          }
          uint8_t* bd = bbuf + bst * kPfBStageBytes;
          const uint32_t sfb_col = tbase + kPfTmemSfb + 20 * bst;
          // B: core matrix (slot t, block b) at t*14*128 + b*128; +256 bytes (+16) per MMA
          const uint64_t bd0 = umma_desc(smem_addr(bd), 128, kTcChunk * 128);
          for (int hf = 0; hf < NH; ++hf, ++n) {
            const int cst = n % kTcCanStages;
            if (!pf_wait(&full_can[cst], (n / kTcCanStages) & 1, abort_flag, &w0)) {
              ok = false;
              break;
            }
            tc_fence_after();
            if (hf == 0)  // the chunk's activation scales, once for both halves
#pragma unroll
              for (int at = 0; at < kPfSfbAtoms; ++at)
                tc_cp_sf(sfb_col + 4 * at, umma_desc(smem_addr(bd + kPfBBytes + 512 * at), 128, 128));
            const uint32_t dcol = tbase + (hf ? kPfTmemUp : 0);
            const uint32_t sfa_col = tbase + kPfTmemSfa + 16 * cst;
            const uint32_t a_col = tbase + kPfTmemA + kTcTmemAStage * cst;
            bool acc = acc_h[hf];
#pragma unroll
            for (int s = 0; s < kTcChunk / 2; ++s) {
              if (s < nbc / 2) {
                const uint32_t sfa_id = 2u * (s & 1);
                const int blk = wb + 2 * s;
                const uint32_t sfb_id = (uint32_t)(blk & 3);
                const uint32_t tsfa = (sfa_col + 4 * (s >> 1)) | (sfa_id << 30);
                const uint32_t tsfb = (sfb_col + 4 * ((blk >> 2) - (wb >> 2))) | (sfb_id << 30);
                mma_mxf4_ts(dcol, a_col + 8 * s, bd0 + (uint64_t)(16 * s), idesc_mxf4(128, N, sfa_id, sfb_id), tsfa,
                            tsfb, acc ? 1u : 0u);
                acc = true;
              }
            }
            acc_h[hf] = acc;
            tc_commit(&empty_can[cst]);
          }
          if (!ok) break;
          tc_commit(&empty_b[bst]);  // both halves' MMAs have read the stage
          ++nbq;
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
    // As in the decode kernel: quadrant q's three warps own M-rows 32q .. 32q+31 and split a
    // chunk's 14 blocks {0-3, 12-13}, {4-7}, {8-11}; payload bytes to 4 TMEM columns per block,
    // the E8M0 bytes of a 4-block atom to one TMEM word.
    const int rw = tc_repack_index(warp);
    const int q = rw / 3, wi = rw - 3 * q;
    const int Gr = 8 * (q >> 1) + (lane & 7), j = 2 * (lane >> 3) + (q & 1);
    const uint32_t taddr_lane = (uint32_t)(32 * q) << 16;
    int n = 0;
    for (int i = c; i < nitems && !*abort_flag; i += G) {
      const int2 it = items[i];
      const int rows = min(128, a.rows_e - 128 * it.y);
      const int gv = rows >= 128 ? 16 : rows / 8;
      const bool row_ok = Gr < gv;
      for (int qc = 0; qc < nq && !*abort_flag; ++qc) {
        for (int hf = 0; hf < NH; ++hf, ++n) {  // the producer's order: (q, gate), (q, up), ..
          const int wb = kTcChunk * qc, nbc = min(kTcChunk, nb - wb);
          const int st = n % kPfRawStages, cst = n % kTcCanStages;
          if (!pf_wait(&full_raw[st], (n / kPfRawStages) & 1, abort_flag, &w0)) break;
          // this lane's row in the staged boxes, as a shared-window address (ld.shared below)
          const uint32_t rs = smem_addr(raw) + st * kTcRawBytes + j * kTcBoxBytes + Gr * kTcBoxW +
                              ((j * rb + 17 * wb) & 15);
          constexpr int kU = 6;
          uint32_t wv[kU][5];
#pragma unroll
          for (int u = 0; u < kU; ++u) {
            const int b = wi == 0 ? (u < 4 ? u : u + 8) : 4 * wi + u;
            const bool ok = row_ok && (wi == 0 || u < 4) && b < nbc;
            const uint32_t wa = (rs + 17 * b) & ~3u;
#pragma unroll
            for (int kk = 0; kk < 5; ++kk) wv[u][kk] = ok ? lds32(wa + 4 * kk) : 0u;
          }
          uint32_t pay[4 * kU], sw[2] = {0u, 0u};
#pragma unroll
          for (int u = 0; u < kU; ++u) {
            const int b = wi == 0 ? (u < 4 ? u : u + 8) : 4 * wi + u;
            const uint32_t a0 = (rs + 17 * b) & 3u;
            const uint32_t sh = 8 * ((a0 + 1) & 3);
            const bool whole = a0 == 3;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              pay[4 * u + kk] = whole ? wv[u][kk + 1] : __funnelshift_r(wv[u][kk], wv[u][kk + 1], sh);
            sw[u >> 2] |= ((wv[u][0] >> (8 * a0)) & 0xFFu) << (8 * (u & 3));
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty_raw[st]);
          if (!pf_wait(&empty_can[cst], ((n / kTcCanStages) & 1) ^ 1, abort_flag, &w1)) break;
          tc_fence_after();
          const uint32_t acol = tbase + kPfTmemA + kTcTmemAStage * cst + taddr_lane;
          const uint32_t scol = tbase + kPfTmemSfa + 16 * cst + q + taddr_lane;
          {
            uint32_t v16[16];
#pragma unroll
            for (int kk = 0; kk < 16; ++kk) v16[kk] = pay[kk];
            tmem_st_x16(acol + 16 * wi, v16);
            tmem_st_x1(scol + 4 * wi, sw[0]);
            if (wi == 0) {
              uint32_t v8[8];
#pragma unroll
              for (int kk = 0; kk < 8; ++kk) v8[kk] = pay[16 + kk];
              tmem_st_x8(acol + 48, v8);
              tmem_st_x1(scol + 12, sw[1]);
            }
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&full_can[cst]);
        }
      }
    }
    if (tr && rw == 0 && lane == 0) {
      tr[kPfEvRepFullRaw] = w0;
      tr[kPfEvRepEmptyCan] = w1;
      tr[kPfEvRepEnd] = globaltimer_ns();
    }
  } else if (tc_epi_quadrant(warp) >= 0) {
    // ================================================================= epilogue warps
    const int q = tc_epi_quadrant(warp);
    const int mrow = 32 * q + lane;
    const int row = tc_row_of(mrow);
    int nit = 0;
    for (int i = c; i < nitems; i += G, ++nit) {
      const int2 it = items[i];
      const int4 g = W.grp[it.x];
      const int ntok = g.z, p0 = g.y;
      const int r = 128 * it.y + row;  // neuron (phase 1) or output row (phase 2)
      const bool valid = r < a.rows_e;
      float b0 = 0.f, b1 = 0.f;
      if (valid) {
        if (a.bias0) b0 = a.bias0[(int64_t)g.x * a.rows_e + r];
        if (PH == 0 && a.bias1) b1 = a.bias1[(int64_t)g.x * a.rows_e + r];
      }
      if (!pf_wait(full_d, nit & 1, abort_flag, &w0)) break;
      const uint64_t tb = tr ? globaltimer_ns() : 0;
      tc_fence_after();
      const uint32_t ta = tbase + ((uint32_t)(32 * q) << 16);
      float vg[kPfGroup], vu[kPfGroup];
#pragma unroll
      for (int tp = 0; tp < kPfGroup / 2; ++tp) {
        vg[2 * tp] = vg[2 * tp + 1] = vu[2 * tp] = vu[2 * tp + 1] = 0.f;
        if (2 * tp < ntok) {
          uint32_t v[16], u[16];
          tmem_ld_x16(ta + 16 * tp, v);
          if (PH == 0) tmem_ld_x16(ta + kPfTmemUp + 16 * tp, u);
          tmem_wait_ld();
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            float sg = 0.f, su = 0.f;
#pragma unroll
            for (int pl = 0; pl < 8; ++pl) {
              sg += __uint_as_float(v[8 * h2 + pl]);
              if (PH == 0) su += __uint_as_float(u[8 * h2 + pl]);
            }
            vg[2 * tp + h2] = sg;
            vu[2 * tp + h2] = su;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(empty_d);
      if (tr) w1 += globaltimer_ns() - tb;
      if (PH == 0) {
#pragma unroll
        for (int t = 0; t < kPfGroup; ++t)
          if (t < ntok)
            xchg[t * 128 + row] = valid ? activate(a.act_mode, vg[t] + b0, vu[t] + b1, a.alpha, a.limit) : 0.f;
        named_sync(1, 128);
        // digit planes of 32-neuron blocks: warp q takes units (t, b) = u / 4, u % 4 for u = q, q+4, ..
        for (int u = q; u < ntok * 4; u += 4) {
          const int t = u >> 2, b = u & 3, blk = 4 * it.y + b;
          if (32 * blk >= a.F) continue;  // whole warps: F is a multiple of 64
          const float av = xchg[t * 128 + 32 * b + lane];
          float m = fabsf(av);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
          const int be = block_be(m);
          const uint32_t cd = digit_planes(av, be);
          const uint32_t hi = __shfl_down_sync(0xffffffffu, cd, 16);
          const int pr = p0 + t;
          if (lane < 16) {
            uint8_t* img = W.planes2 + ((size_t)pr * (a.F / 32) + blk) * 128;
#pragma unroll
            for (int pl = 0; pl < 8; ++pl)
              img[pl * 16 + lane] = (uint8_t)(((cd >> (4 * pl)) & 15u) | (((hi >> (4 * pl)) & 15u) << 4));
          } else if (lane < 24) {
            const int pl = lane - 16;
            W.sf2[(size_t)it.x * W.sf2_bytes + (blk >> 2) * 512 + pf_sf_byte(t, pl, blk)] = (uint8_t)plane_scale(pl, be);
          }
        }
        named_sync(1, 128);
      } else {
#pragma unroll
        for (int t = 0; t < kPfGroup; ++t)
          if (t < ntok) xchg[t * 128 + row] = vg[t] + b0;
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
  if (!al16(p->gate_w) || !al16(p->up_w) || !al16(p->down_w) || !al16(p->x) || !al16(p->out))
    return fail(NS_ERR_INVALID, "ns_moe_prefill_grouped: expert tensors, x and out must be 16-byte aligned");
  const int64_t P = (int64_t)p->T * p->k;
  const int nl = p->expert_hi - p->expert_lo;
  pl->P = (int)P;
  pl->Gmax = (int)std::min<int64_t>(P, (P + kPfGroup - 1) / kPfGroup + nl);
  pl->ns1 = (p->F + 127) / 128;
  pl->nr2 = (p->H + 127) / 128;
  pl->nb_h = p->H / 32;
  pl->nb_f = p->F / 32;
  pl->sf1_bytes = ((pl->nb_h + 3) / 4 + 4) * 512;
  pl->sf2_bytes = ((pl->nb_f + 3) / 4 + 4) * 512;
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

// Planes of `P` pairs x `nb` blocks x 128 bytes as a 3-D u32 tensor; box = 16 pairs x 14 blocks.
static int make_planes_map(CUtensorMap* m, const uint8_t* base, int P, int nb) {
  EncodeTiledFn fn;
  int st = get_encode_fn(&fn);
  if (st) return st;
  const cuuint64_t dims[3] = {32, (cuuint64_t)nb, (cuuint64_t)P};
  const cuuint64_t strides[2] = {128, (cuuint64_t)nb * 128};
  const cuuint32_t box[3] = {32, (cuuint32_t)kTcChunk, (cuuint32_t)kPfGroup};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<uint8_t*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NS_ERR_CUDA, "cuTensorMapEncodeTiled (planes) failed (%d)", (int)r);
  return NS_OK;
}

static size_t pf_gemm_smem(PfGemmArgs* a) {
  size_t off = 0;
  a->off_raw = 0;
  off += (size_t)kPfRawStages * kTcRawBytes;
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
  pf_logits_kernel<<<dim3((p->T + kPfLgT - 1) / kPfLgT, (p->n_expert + kPfLgE - 1) / kPfLgE), 128, 0, s>>>(*p, w,
                                                                                                       logits);
  NS_CUDA_TRY(cudaGetLastError());
  pf_topk_kernel<<<(p->T + 7) / 8, 256, 0, s>>>(*p, w, logits);
  NS_CUDA_TRY(cudaGetLastError());
  // 2. bucket (ids staged in shared memory when they fit)
  const size_t ids_bytes = (size_t)p->T * p->k * 4;
  const bool ids_smem = ids_bytes <= (size_t)kPfBucketSmem;
  NS_CUDA_TRY(cudaFuncSetAttribute(pf_bucket_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPfBucketSmem));
  pf_bucket_kernel<<<1, 1024, ids_smem ? ids_bytes : 0, s>>>(*p, w, pl.ns1, pl.nr2, ids_smem ? 1 : 0);
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
  const int nl = p->expert_hi - p->expert_lo;
  const int rb_h = (int)row_bytes_of(p->ggml_type, p->H), rb_f = (int)row_bytes_of(p->ggml_type, p->F);
  {
    const int64_t rows = (int64_t)nl * p->F;
    st = make_row_group_map(&a.tm_a16[0], p->gate_w, rows, rb_h, 16);
    if (!st) st = make_row_group_map(&a.tm_a8[0], p->gate_w, rows, rb_h, 8);
    if (!st) st = make_row_group_map(&a.tm_a16[1], p->up_w, rows, rb_h, 16);
    if (!st) st = make_row_group_map(&a.tm_a8[1], p->up_w, rows, rb_h, 8);
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
    st = make_row_group_map(&a.tm_a16[0], p->down_w, rows, rb_f, 16);
    if (!st) st = make_row_group_map(&a.tm_a8[0], p->down_w, rows, rb_f, 8);
    if (!st) st = make_planes_map(&a.tm_b, w.planes2, pl.P, pl.nb_f);
    if (st) return st;
    a.tm_a16[1] = a.tm_a16[0];
    a.tm_a8[1] = a.tm_a8[0];
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
