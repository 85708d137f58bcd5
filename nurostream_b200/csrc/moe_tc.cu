// Fused MoE decode layer on the tcgen05 tensor cores (MXFP4 experts, T <= 2).
//
// Same contract and results (to fp32 rounding) as moe_layer_kernel in moe.cu;
// ns_moe_decode_layer picks this kernel when the layer qualifies
// (moe_tc_eligible).  One cooperative launch, one CTA per SM.
//
// Arithmetic.  Every expert projection is D[row, plane] = sum_k W[row, k] *
// P[plane, k] on `tcgen05.mma.kind::mxf4.block_scale.block32`:
//   * A (M = 128) is 128 weight rows, copied from the GGUF bytes: the 16
//     payload bytes of an MXFP4 block become one 16-byte row of a core matrix
//     as they are, and its E8M0 byte becomes the row's UE8M0 block scale
//     (GGML's value table[code] * 2^(e-128) equals the OCP MX value
//     e2m1[code] * 2^(e-127)).  GGUF packs element j in the low nibble and
//     element j+16 in the high nibble of byte j, so the MMA's K order is the
//     block's elements (0,16,1,17,...); the activation planes use the same
//     order, which leaves every dot product unchanged.
//   * B (N = 8 per token) holds the activation as 8 balanced radix-8 digit
//     planes: per 32-element block with max |v| < 2^e, v = sum_p d_p 8^p
//     2^(e-23) with integer digits d_p in [-4, 4] (an exact 24-bit fixed-point
//     split), and digit d is the e2m1 value d/2 with block scale 2^(3p+e-22).
//   * D accumulates in fp32 in TMEM; the epilogue adds the 8 plane columns.
//
// Work.  Phase 1 tiles are 64-neuron slabs of one routed expert (64 gate rows
// + 64 up rows = M); phase 2 tiles are 128 down rows of one (token, expert)
// pair.  The concatenated K-blocks of all tiles are split evenly over the CTAs
// at 8-block chunk boundaries ("stream-K"), so every SM streams the same
// number of weight bytes.  A tile split over CTAs is finished by the last one
// to arrive (fixed summation order, so results are deterministic).  Phase 2
// of expert e starts as soon as all slabs of e are done (per-expert counters);
// the combine of a row block runs when all of its pairs are done.  No grid
// barrier follows the routing barrier.
//
// Warps: 0 producer (TMA), 1 MMA issuer, 2..9 repack raw rows into the
// operand layout, 10..13 epilogue (TMEM -> registers, finish tiles).  Every
// wait is bounded; a wait that runs out raises a device error bit, stops the
// CTA's pipeline, lets in-flight copies and MMAs land, frees TMEM and returns.

#include "tc.cuh"

namespace ns {

constexpr int kTcWarps = 14;
constexpr int kTcThreads = kTcWarps * 32;
constexpr int kTcRepackWarp0 = 2, kTcRepackWarps = 8, kTcEpiWarp0 = 10;
constexpr int kTcRawStages = 4, kTcCanStages = 3;
constexpr int kTcChunk = 8;                          // K blocks (32 elements) per chunk
constexpr int kTcBoxW = 160;                         // TMA box width (bytes): >= 8*17 + 14, multiple of 16
constexpr int kTcBoxBytes = kTcBoxW * 8;             // 8 row groups per box
constexpr int kTcRawBytes = 16 * kTcBoxBytes;        // 2 halves x 8 row phases
constexpr int kTcCanA = 16 * kTcChunk * 128;         // 16 row groups x 8 blocks x 128 B
constexpr int kTcCanSFA = 2 * 512;
constexpr int kTcCanB = kTcChunk * 128;              // phase-2 B: 8 planes x 8 blocks
constexpr int kTcCanSFB = 2 * 512;
constexpr int kTcCanBytes = kTcCanA + kTcCanSFA + kTcCanB + kTcCanSFB;
constexpr int kTcTmemCols = 128;                     // D: 2 x 16 cols; SF: 3 stages x 16 cols
constexpr int kTcMaxSegs = 8;                        // tiles one CTA touches
constexpr int kTcMaxSplit = 16;                      // CTAs one tile is split over
constexpr int kTcMaxTiles = 2048;
constexpr int kTcWsHeader = 16384;                   // barrier word, counters
constexpr int kTcOffCnt = 1024, kTcOffReady = 1024 + 4 * kTcMaxTiles, kTcOffCnt2 = kTcOffReady + 4 * 128;
constexpr int kTcMaxRowTiles = (kTcWsHeader - kTcOffCnt2) / 4;
constexpr int kTcSmemBudget = 225 * 1024;

struct MoeTcArgs {
  CUtensorMap tm_gate, tm_up, tm_down;  // 8-row groups x 8*row_bytes bytes, box 160 x 8
  ns_moe_layer_t p;
  int rb_h, rb_f, nb_h, nb_f;
  unsigned long long* bar;
  unsigned* cnt;     // per tile: segments finished
  unsigned* ready;   // per slot: phase-1 slabs finished
  unsigned* cnt2;    // per phase-2 row tile: pairs finished
  float* logits;     // T x E
  float* partial;    // [G][2][T][128]
  uint8_t* actimg;   // per pair: planes [nb_f][8][16] then scales [nb_f][8]
  float* yp;         // per pair: H fp32
  int img_bytes;
  int zero_tiles;    // counters to clear per launch
  int off_raw, off_b1, off_sfb1, off_can, off_xchg, off_bars, off_shared;
  int sfb1_atom;     // bytes between phase-1 scale atoms (128 * T)
  unsigned long long* trace;
};

struct TcSeg {
  int tile, k0, k1;            // K blocks [k0, k1) of the tile
  int nsplit;                  // CTAs sharing the tile
  short split_cta[kTcMaxSplit];
  char split_slot[kTcMaxSplit];
  int my_slot;                 // this CTA's partial slot (0 first segment, 1 last)
};

struct TcShared {
  int ids[NS_MAX_TOKENS][NS_MAX_TOPK];
  float w[NS_MAX_TOKENS][NS_MAX_TOPK];
  float topv[NS_MAX_TOKENS][NS_MAX_TOPK];
  float rscale[NS_MAX_TOKENS];
  float red[kTcWarps][NS_MAX_TOKENS];
  float red2[kTcWarps][NS_MAX_TOKENS];
  int nslots, npairs;
  int slot_expert[kMaxPairs];
  int slot_pair0[kMaxPairs + 1];
  int pair_token[kMaxPairs];
  int pair_slot[kMaxPairs];
  float pair_w[kMaxPairs];
  unsigned long long bar_target;
  int ok;
  int abort_flag;
  uint32_t tmem_base;
  int nseg;
  TcSeg seg[kTcMaxSegs];
  int fin;
  int bnd[1025];  // CTA range boundaries in K blocks (grid <= 1024)
  __align__(16) float scratch[NS_MAX_EXPERTS];
};

// Geometry of the tile list: phase-1 slabs (slot-major), then phase-2 row tiles (pair-major).
struct TcGeom {
  int T1, T2, ns1, nr2, nb_h, nb_f;
  __device__ int64_t start(int i) const {
    return i < T1 ? (int64_t)i * nb_h : (int64_t)T1 * nb_h + (int64_t)(i - T1) * nb_f;
  }
  __device__ int len(int i) const { return i < T1 ? nb_h : nb_f; }
  __device__ int tile_of(int64_t u) const {
    const int64_t u1 = (int64_t)T1 * nb_h;
    return u < u1 ? (int)(u / nb_h) : T1 + (int)((u - u1) / nb_f);
  }
  __device__ int64_t total() const { return (int64_t)T1 * nb_h + (int64_t)T2 * nb_f; }
};

__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      raise_device_error(NS_DEVERR_COPY_WAIT);
      *abort_flag = 1;
      return false;
    }
  }
  return true;
}

// e2m1 code of digit d in [-4, 4] (value d/2): magnitude |d| is the code, bit 3 the sign.
__device__ __forceinline__ uint32_t digit_code(int d) { return (uint32_t)(d < 0 ? (8 - d) : d); }

// Balanced radix-8 split of one value given its block exponent e (max|v| < 2^e):
// nibble codes of the 8 planes packed in a 32-bit word (plane p in bits 4p..4p+3).
__device__ __forceinline__ uint32_t digit_planes(float v, int e) {
  int X = (int)rintf(ldexpf(v, 23 - e));
  uint32_t codes = 0;
#pragma unroll
  for (int p = 0; p < 7; ++p) {
    int d = X & 7;
    d = d > 4 ? d - 8 : d;
    X = (X - d) >> 3;
    codes |= digit_code(d) << (4 * p);
  }
  return codes | (digit_code(X) << 28);
}

// E8M0 scale byte of plane p for block exponent e (block all zero: any scale).
__device__ __forceinline__ uint32_t plane_scale(int p, int e, bool nonzero) {
  if (!nonzero) return 127u;
  const int s = 3 * p + e + 105;
  return (uint32_t)(s < 0 ? 0 : (s > 254 ? 254 : s));
}

// Block exponent: max|v| < 2^e.
__device__ __forceinline__ int block_exp(float m) {
  int e = 0;
  if (m > 0.f) frexpf(m, &e);
  return e;
}

// One half-warp (16 lanes, lane j holds block values v[j] and v[j+16]) writes the
// 8 planes of one block: plane p byte j = code(v[j]) | code(v[j+16]) << 4, to
// dst + p*16 + j; the 8 scale bytes to sdst[p * sstride] (lane 0 of the half).
__device__ __forceinline__ void halfwarp_block_planes(float v0, float v1, uint8_t* dst, uint8_t* sdst, int sstride,
                                                      int hl /*0..15*/, unsigned mask) {
  float m = fmaxf(fabsf(v0), fabsf(v1));
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(mask, m, o, 16));
  const int e = block_exp(m);
  const bool nz = m > 0.f;
  const uint32_t c0 = nz ? digit_planes(v0, e) : 0u, c1 = nz ? digit_planes(v1, e) : 0u;
#pragma unroll
  for (int p = 0; p < 8; ++p) {
    const uint32_t b = ((c0 >> (4 * p)) & 15u) | (((c1 >> (4 * p)) & 15u) << 4);
    dst[p * 16 + hl] = (uint8_t)b;
  }
  if (hl == 0)
#pragma unroll
    for (int p = 0; p < 8; ++p) sdst[p * sstride] = (uint8_t)plane_scale(p, e, nz);
}

template <int NT>
__global__ void __launch_bounds__(kTcThreads, 1) moe_tc_kernel(const __grid_constant__ MoeTcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const ns_moe_layer_t& p = a.p;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, c = blockIdx.x;
  const int T = NT, H = p.H, F = p.F, E = p.n_expert, k = p.k;

  uint8_t* raw = smem + a.off_raw;
  uint8_t* b1 = smem + a.off_b1;
  uint8_t* sfb1 = smem + a.off_sfb1;
  uint8_t* can = smem + a.off_can;
  float* xchg = reinterpret_cast<float*>(smem + a.off_xchg);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + a.off_bars);
  uint64_t* full_raw = bars;
  uint64_t* empty_raw = full_raw + kTcRawStages;
  uint64_t* full_can = empty_raw + kTcRawStages;
  uint64_t* empty_can = full_can + kTcCanStages;
  uint64_t* full_d = empty_can + kTcCanStages;
  uint64_t* empty_d = full_d + 2;
  uint64_t* mma_done = empty_d + 2;
  TcShared& S = *reinterpret_cast<TcShared*>(smem + a.off_shared);
  volatile int* abort_flag = &S.abort_flag;

  if (tid == 0) {
    stamp(a.trace, kEvStart);
    for (int s = 0; s < kTcRawStages; ++s) {
      mbar_init(&full_raw[s], 1);
      mbar_init(&empty_raw[s], kTcRepackWarps);
    }
    for (int s = 0; s < kTcCanStages; ++s) {
      mbar_init(&full_can[s], kTcRepackWarps);
      mbar_init(&empty_can[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&full_d[s], 1);
      mbar_init(&empty_d[s], 4);
    }
    mbar_init(mma_done, 1);
    fence_mbar_init();
    // TMA boxes and operand tiles assume a 1024-byte aligned dynamic shared-memory base
    S.abort_flag = (smem_addr(smem) & 1023u) != 0;
    if (S.abort_flag) raise_device_error(NS_DEVERR_COPY_WAIT);
    prefetch_tmap(&a.tm_gate);
    prefetch_tmap(&a.tm_up);
    prefetch_tmap(&a.tm_down);
  }
  if (warp == 1) tmem_alloc(&S.tmem_base, kTcTmemCols);
  // counters of this launch (used only after the routing barrier)
  if (c == 0) {
    for (int i = tid; i < a.zero_tiles; i += kTcThreads) a.cnt[i] = 0u;
    for (int i = tid; i < kMaxPairs; i += kTcThreads) a.ready[i] = 0u;
    for (int i = tid; i < kTcMaxRowTiles; i += kTcThreads) a.cnt2[i] = 0u;
  }

  // ---- 1. x into shared memory, RMSNorm sum of squares, this CTA's router logit
  float* h = reinterpret_cast<float*>(raw);  // T x H fp32, reused by the raw ring after the prologue
  const bool own_expert = c < E;
  for (int t = 0; t < T; ++t) {
    float ss = 0.f, dot = 0.f;
    for (int i = tid; i < H; i += kTcThreads) {
      const float xv = p.x[(int64_t)t * H + i];
      const float wv = p.norm_w ? p.norm_w[i] : 1.0f;
      const float rv = own_expert ? load_float(p.router_w, p.router_dtype, (int64_t)c * H + i) : 0.f;
      h[t * H + i] = xv;
      ss = fmaf(xv, xv, ss);
      dot = fmaf(xv * wv, rv, dot);
    }
    ss = warp_sum(ss);
    dot = warp_sum(dot);
    if (lane == 0) {
      S.red[warp][t] = ss;
      S.red2[warp][t] = dot;
    }
  }
  __syncthreads();
  if (tid < T) {
    float ss = 0.f, dot = 0.f;
    for (int w = 0; w < kTcWarps; ++w) {
      ss += S.red[w][tid];
      dot += S.red2[w][tid];
    }
    const float r = p.norm_w ? 1.0f / sqrtf(ss / (float)H + p.rms_eps) : 1.0f;
    S.rscale[tid] = r;
    if (own_expert) a.logits[(int64_t)tid * E + c] = r * dot + (p.router_b ? p.router_b[c] : 0.f);
  }
  __syncthreads();
  if (p.norm_w)
    for (int t = 0; t < T; ++t) {
      const float r = S.rscale[t];
      for (int i = tid; i < H; i += kTcThreads) h[t * H + i] = __fmul_rn(__fmul_rn(h[t * H + i], r), p.norm_w[i]);
    }
  __syncthreads();
  if (tid == 0) stamp(a.trace, kEvNorm);
  for (int e = c + G; e < E; e += G) {  // more experts than CTAs
    float sacc[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) sacc[t] = 0.f;
    for (int i = tid; i < H; i += kTcThreads) {
      const float wv = load_float(p.router_w, p.router_dtype, (int64_t)e * H + i);
#pragma unroll
      for (int t = 0; t < NT; ++t) sacc[t] = fmaf(h[t * H + i], wv, sacc[t]);
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const float v = warp_sum(sacc[t]);
      if (lane == 0) S.red[warp][t] = v;
    }
    __syncthreads();
    if (tid < T) {
      float v = 0.f;
      for (int w = 0; w < kTcWarps; ++w) v += S.red[w][tid];
      a.logits[(int64_t)tid * E + e] = v + (p.router_b ? p.router_b[e] : 0.f);
    }
    __syncthreads();
  }

  // ---- 2. split-phase grid barrier around the build of the phase-1 activation planes
  if (tid == 0) {
    stamp(a.trace, kEvRouter);
    __threadfence();
    const unsigned long long old = atomicAdd(a.bar, 1ull);
    S.bar_target = (old / (unsigned)G + 1ull) * (unsigned)G;
  }
  {
    // B1: token t's planes are rows 8t..8t+7; core matrix (t, block b) at t*nb_h*128 + b*128.
    // SFB1: atom b/4 at (b/4)*sfb1_atom, byte 16*(8t+p) + b%4.
    const int nb = a.nb_h;
    const int half = (tid >> 4), hl = tid & 15;
    const unsigned mask = 0xFFFFu << (lane & 16);
    for (int it = half; it < T * nb; it += kTcThreads / 16) {
      const int t = it / nb, b = it - t * nb;
      const float* hv = h + t * H + 32 * b;
      uint8_t* dst = b1 + (size_t)t * nb * 128 + b * 128;
      uint8_t* sdst = sfb1 + (b >> 2) * a.sfb1_atom + 16 * (8 * t) + (b & 3);
      halfwarp_block_planes(hv[hl], hv[hl + 16], dst, sdst, 16, hl, mask);
    }
  }
  if (tid == 0) {
    S.ok = 1;
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_u64(a.bar) < S.bar_target) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        raise_device_error(NS_DEVERR_GRID_WAIT);
        S.ok = 0;
        S.abort_flag = 1;
        break;
      }
      __nanosleep(32);
    }
    stamp(a.trace, kEvBarrier1);
  }
  __syncthreads();

  // ---- 3. routing (every CTA, identical): rank of each expert by (score desc, index asc)
  float* sc_e = S.scratch;
  for (int t = 0; t < T; ++t) {
    float m = -INFINITY;
    for (int e = tid; e < E; e += kTcThreads) {
      const float lg = __ldcg(a.logits + (int64_t)t * E + e);
      sc_e[e] = lg;
      m = fmaxf(m, lg);
    }
    if (p.route_mode == NS_ROUTE_SOFTMAX_TOPK_NORM) {
      // softmax over all experts first (neurostream/moe/router.py:64-65)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (lane == 0) S.red[warp][0] = m;
      __syncthreads();
      m = S.red[0][0];
      for (int w = 1; w < kTcWarps; ++w) m = fmaxf(m, S.red[w][0]);
      float sum = 0.f;
      for (int e = tid; e < E; e += kTcThreads) {
        const float ex = expf(sc_e[e] - m);
        sc_e[e] = ex;
        sum += ex;
      }
      sum = warp_sum(sum);
      __syncthreads();
      if (lane == 0) S.red[warp][0] = sum;
      __syncthreads();
      sum = 0.f;
      for (int w = 0; w < kTcWarps; ++w) sum += S.red[w][0];
      for (int e = tid; e < E; e += kTcThreads) sc_e[e] = sc_e[e] / sum;
    }
    __syncthreads();
    for (int e = tid; e < E; e += kTcThreads) {
      const float score = sc_e[e];
      int rank = 0, e2 = 0;
      for (; e2 + 4 <= E; e2 += 4) {
        const float4 v4 = *reinterpret_cast<const float4*>(sc_e + e2);
        rank += (v4.x > score || (v4.x == score && e2 < e));
        rank += (v4.y > score || (v4.y == score && e2 + 1 < e));
        rank += (v4.z > score || (v4.z == score && e2 + 2 < e));
        rank += (v4.w > score || (v4.w == score && e2 + 3 < e));
      }
      for (; e2 < E; ++e2) rank += (sc_e[e2] > score || (sc_e[e2] == score && e2 < e));
      if (rank < k) {
        S.ids[t][rank] = e;
        S.topv[t][rank] = score;
      }
    }
    __syncthreads();
    if (warp == 0) {
      const float v = lane < k ? S.topv[t][lane] : 0.f;
      float wgt;
      if (p.route_mode == NS_ROUTE_TOPK_SOFTMAX) {
        // softmax over the k (neurostream/model/gpt_oss.py:119-120)
        const float mx = S.topv[t][0];
        const float ex = lane < k ? expf(v - mx) : 0.f;
        wgt = ex / warp_sum(ex);
      } else {
        wgt = v / warp_sum(v);  // renormalise the top-k probabilities (router.py:66-68)
      }
      if (lane < k) S.w[t][lane] = wgt;
    }
    __syncthreads();
  }
  if (tid == 0) stamp(a.trace, kEvTopk);

  // ---- 4. slots (distinct local experts, ascending) and pairs (slot-major, token ascending)
  if (tid == 0) {
    int n = 0;
    for (int t = 0; t < T; ++t)
      for (int j = 0; j < k; ++j) {
        const int e = S.ids[t][j];
        if (e < p.expert_lo || e >= p.expert_hi) continue;
        bool seen = false;
        for (int q = 0; q < n; ++q) seen |= S.slot_expert[q] == e;
        if (!seen) S.slot_expert[n++] = e;
      }
    for (int i = 1; i < n; ++i) {  // insertion sort, n <= T*k
      const int v = S.slot_expert[i];
      int j = i - 1;
      while (j >= 0 && S.slot_expert[j] > v) {
        S.slot_expert[j + 1] = S.slot_expert[j];
        --j;
      }
      S.slot_expert[j + 1] = v;
    }
    int np = 0;
    for (int s = 0; s < n; ++s) {
      S.slot_pair0[s] = np;
      for (int t = 0; t < T; ++t)
        for (int j = 0; j < k; ++j)
          if (S.ids[t][j] == S.slot_expert[s]) {
            S.pair_token[np] = t;
            S.pair_w[np] = S.w[t][j];
            S.pair_slot[np] = s;
            ++np;
          }
    }
    S.slot_pair0[n] = np;
    S.nslots = n;
    S.npairs = np;
  }
  if (c == 0 && warp == 0)
    for (int i = lane; i < T * k; i += 32) {
      if (p.ids) p.ids[i] = S.ids[i / k][i % k];
      if (p.weights) p.weights[i] = S.w[i / k][i % k];
    }
  __syncthreads();

  TcGeom geo;
  geo.ns1 = F / 64;
  geo.nr2 = (H + 127) / 128;
  geo.T1 = S.nslots * geo.ns1;
  geo.T2 = S.npairs * geo.nr2;
  geo.nb_h = a.nb_h;
  geo.nb_f = a.nb_f;
  const int64_t U = geo.total();

  // ---- 5. CTA ranges (K blocks, snapped to chunk boundaries) and this CTA's segments
  for (int j = tid; j <= G; j += kTcThreads) {
    int64_t b;
    if (j == G || U == 0) {
      b = j == G ? U : 0;
    } else {
      const int64_t u = U * j / G;
      const int i = geo.tile_of(u);
      const int64_t s0 = geo.start(i);
      const int L = geo.len(i);
      const int off = (int)(u - s0);
      b = s0 + min(L, ((off + kTcChunk / 2) / kTcChunk) * kTcChunk);
    }
    S.bnd[j] = (int)b;
  }
  __syncthreads();
  if (tid == 0) {
    int ns = 0;
    int64_t u = S.bnd[c];
    const int64_t uend = S.bnd[c + 1];
    while (u < uend && ns < kTcMaxSegs) {
      const int i = geo.tile_of(u);
      const int64_t s0 = geo.start(i), e0 = s0 + geo.len(i);
      TcSeg& sg = S.seg[ns];
      sg.tile = i;
      sg.k0 = (int)(u - s0);
      sg.k1 = (int)(min(e0, uend) - s0);
      sg.my_slot = ns == 0 ? 0 : 1;
      // CTAs sharing tile i, ascending: first one whose range contains s0, then on while ranges start before e0
      int lo = 0, hi = G - 1;
      while (lo < hi) {  // largest cc with bnd[cc] <= s0
        const int mid = (lo + hi + 1) >> 1;
        if (S.bnd[mid] <= s0) lo = mid; else hi = mid - 1;
      }
      int nsp = 0;
      for (int cc = lo; cc < G && S.bnd[cc] < e0; ++cc) {
        if (S.bnd[cc + 1] <= S.bnd[cc] || S.bnd[cc + 1] <= s0) continue;  // empty or before the tile
        if (nsp < kTcMaxSplit) {
          sg.split_cta[nsp] = (short)cc;
          sg.split_slot[nsp] = (char)(S.bnd[cc] >= s0 ? 0 : 1);
        }
        ++nsp;
      }
      sg.nsplit = nsp;
      if (nsp > kTcMaxSplit) {
        raise_device_error(NS_DEVERR_ROUTE);
        S.abort_flag = 1;
      }
      u = e0 < uend ? e0 : uend;
      ++ns;
    }
    if (u < uend) {
      raise_device_error(NS_DEVERR_ROUTE);
      S.abort_flag = 1;
    }
    S.nseg = ns;
    stamp(a.trace, kEvRoute);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  const int nseg = S.nseg;
  const uint32_t tbase = S.tmem_base;

  // ---- no routed local expert (expert parallel): this rank contributes zeros (+ residual)
  if (S.npairs == 0) {
    const int r0 = (int)((int64_t)H * c / G), r1 = (int)((int64_t)H * (c + 1) / G);
    for (int q = tid; q < T * (r1 - r0); q += kTcThreads) {
      const int t = q / (r1 - r0), r = r0 + (q - t * (r1 - r0));
      p.out[(int64_t)t * H + r] = p.add_residual ? p.x[(int64_t)t * H + r] : 0.f;
    }
  } else if (warp == 0) {
    // ================================================================= producer (TMA)
    if (lane == 0) {
      int n = 0;
      for (int sgi = 0; sgi < nseg && !*abort_flag; ++sgi) {
        const TcSeg sg = S.seg[sgi];
        const int i = sg.tile;
        const bool ph1 = i < geo.T1;
        const int rb = ph1 ? a.rb_h : a.rb_f;
        int y0, nh;
        const CUtensorMap *tm0, *tm1;
        if (ph1) {
          const int sl = i % geo.ns1, el = S.slot_expert[i / geo.ns1] - p.expert_lo;
          y0 = (el * F + 64 * sl) / 8;
          nh = 2;
          tm0 = &a.tm_gate;
          tm1 = &a.tm_up;
        } else {
          const int q = i - geo.T1, pp = q / geo.nr2, rt = q % geo.nr2;
          const int el = S.slot_expert[S.pair_slot[pp]] - p.expert_lo;
          y0 = (el * H + 128 * rt) / 8;
          nh = (H - 128 * rt) >= 128 ? 2 : 1;
          tm0 = &a.tm_down;
          tm1 = &a.tm_down;
        }
        for (int kb = sg.k0; kb < sg.k1 && !*abort_flag; kb += kTcChunk, ++n) {
          const int st = n % kTcRawStages;
          if (!tc_wait(&empty_raw[st], ((n / kTcRawStages) & 1) ^ 1, abort_flag)) break;
          mbar_arrive_expect_tx(&full_raw[st], (uint32_t)(nh * 8 * kTcBoxBytes));
          uint8_t* dst = raw + st * kTcRawBytes;
          const int cc = kb / kTcChunk;
          for (int hh = 0; hh < nh; ++hh) {
            const CUtensorMap* tm = hh == 0 ? tm0 : tm1;
            const int yy = ph1 ? y0 : y0 + 8 * hh;
#pragma unroll 1
            for (int j = 0; j < 8; ++j) {
              const int x0 = (j * rb + cc * 136) & ~15;
              tma_load_2d(dst + (hh * 8 + j) * kTcBoxBytes, tm, x0, yy, &full_raw[st]);
            }
          }
          if (n == 0) stamp(a.trace, kEvProducerFirst);
        }
      }
      // let every issued load land before the CTA can exit
      for (int q = max(0, n - kTcRawStages); q < n; ++q)
        mbar_wait_bounded(&full_raw[q % kTcRawStages], (q / kTcRawStages) & 1);
      stamp(a.trace, kEvProducerLast);
    }
  } else if (warp == 1) {
    // ================================================================= MMA issuer
    if (lane == 0) {
      int n = 0;
      const uint32_t idesc_full1 = idesc_mxf4(128, 8 * NT, 0, 0);
      const uint32_t idesc_full2 = idesc_mxf4(128, 8, 0, 0);
      for (int sgi = 0; sgi < nseg && !*abort_flag; ++sgi) {
        const TcSeg sg = S.seg[sgi];
        const bool ph1 = sg.tile < geo.T1;
        const int db = sgi & 1;
        if (!tc_wait(&empty_d[db], ((sgi >> 1) & 1) ^ 1, abort_flag)) break;
        const uint32_t tmem_d = tbase + 16 * db;
        bool first = true;
        for (int kb = sg.k0; kb < sg.k1; kb += kTcChunk, ++n) {
          const int st = n % kTcCanStages;
          if (!tc_wait(&full_can[st], (n / kTcCanStages) & 1, abort_flag)) break;
          tc_fence_after();
          const int nbc = min(kTcChunk, sg.k1 - kb), cc = kb / kTcChunk;
          uint8_t* cs = can + st * kTcCanBytes;
          const uint32_t sf_col = tbase + 32 + 16 * st;
          for (int at = 0; at < (nbc + 3) / 4; ++at) {
            tc_cp_sf(sf_col + 4 * at, umma_desc(smem_addr(cs + kTcCanA + at * 512), 128, 128));
            const uint8_t* sfb_src = ph1 ? sfb1 + (2 * cc + at) * a.sfb1_atom : cs + kTcCanA + kTcCanSFA + kTcCanB + at * 512;
            tc_cp_sf(sf_col + 8 + 4 * at, umma_desc(smem_addr(sfb_src), 128, 128));
          }
          for (int s = 0; s < nbc / 2; ++s) {
            const uint64_t da = umma_desc(smem_addr(cs + 2 * s * 128), 128, kTcChunk * 128);
            const uint64_t dbd = ph1 ? umma_desc(smem_addr(b1 + (size_t)(kb + 2 * s) * 128), 128, a.nb_h * 128)
                                     : umma_desc(smem_addr(cs + kTcCanA + kTcCanSFA + 2 * s * 128), 128, 1024);
            const uint32_t sfid = 2u * (s & 1);
            const uint32_t id = (ph1 ? idesc_full1 : idesc_full2) | (sfid << 4) | (sfid << 29);
            const uint32_t tsfa = (sf_col + 4 * (s >> 1)) | (sfid << 30);
            const uint32_t tsfb = (sf_col + 8 + 4 * (s >> 1)) | (sfid << 30);
            mma_mxf4(tmem_d, da, dbd, id, tsfa, tsfb, first ? 0u : 1u);
            first = false;
          }
          tc_commit(&empty_can[st]);
        }
        tc_commit(&full_d[db]);
      }
      tc_commit(mma_done);
      mbar_wait_bounded(mma_done, 0);
    }
  } else if (warp < kTcEpiWarp0) {
    // ================================================================= repack warps
    const int rw = warp - kTcRepackWarp0;  // 0..7
    const int j = lane & 7, qd = lane >> 3;
    int n = 0;
    int ready_slot = -1;
    for (int sgi = 0; sgi < nseg && !*abort_flag; ++sgi) {
      const TcSeg sg = S.seg[sgi];
      const int i = sg.tile;
      const bool ph1 = i < geo.T1;
      const int rb = ph1 ? a.rb_h : a.rb_f;
      int gvalid = 16, pp = 0;
      if (!ph1) {
        const int q = i - geo.T1, rt = q % geo.nr2;
        pp = q / geo.nr2;
        gvalid = (H - 128 * rt) >= 128 ? 16 : 8;
        const int slot = S.pair_slot[pp];
        if (slot != ready_slot) {  // this pair's activation planes must be complete (every lane acquires)
          const unsigned target = (unsigned)geo.ns1;
          const uint64_t t0 = globaltimer_ns();
          while (ld_acquire_u32(a.ready + slot) < target) {
            if (*abort_flag) break;
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
              if (lane == 0) raise_device_error(NS_DEVERR_GRID_WAIT);
              *abort_flag = 1;
              break;
            }
            __nanosleep(64);
          }
          __syncwarp();
          ready_slot = slot;
        }
      }
      for (int kb = sg.k0; kb < sg.k1; kb += kTcChunk, ++n) {
        const int st = n % kTcRawStages, cst = n % kTcCanStages;
        if (!tc_wait(&full_raw[st], (n / kTcRawStages) & 1, abort_flag)) break;
        if (!tc_wait(&empty_can[cst], ((n / kTcCanStages) & 1) ^ 1, abort_flag)) break;
        const int nbc = min(kTcChunk, sg.k1 - kb), cc = kb / kTcChunk;
        const uint8_t* rs = raw + st * kTcRawBytes;
        uint8_t* cs = can + cst * kTcCanBytes;
        const int oj = (j * rb + cc * 136) & 15;
        for (int item = rw; item < 32; item += kTcRepackWarps) {
          const int Gr = item >> 1, tt = item & 1;
          if (Gr >= gvalid) continue;
          const int b = (qd + 2 * j + 4 * tt) & 7;
          if (b >= nbc) continue;
          const int hh = Gr >> 3, g = Gr & 7;
          const uint8_t* src = rs + (hh * 8 + j) * kTcBoxBytes + g * kTcBoxW + oj + 17 * b;  // scale byte
          const uint32_t* w = reinterpret_cast<const uint32_t*>(reinterpret_cast<uintptr_t>(src) & ~uintptr_t(3));
          const uint32_t a0 = (uint32_t)(reinterpret_cast<uintptr_t>(src) & 3);
          uint32_t wv[5];
#pragma unroll
          for (int q = 0; q < 5; ++q) wv[q] = w[q];
          const uint32_t scale = (wv[0] >> (8 * a0)) & 0xFFu;
          const uint32_t s1 = a0 + 1;  // payload offset from the first word, 1..4
          uint4 pl;
          if (s1 < 4) {
            const uint32_t sh = 8 * s1;
            pl.x = __funnelshift_r(wv[0], wv[1], sh);
            pl.y = __funnelshift_r(wv[1], wv[2], sh);
            pl.z = __funnelshift_r(wv[2], wv[3], sh);
            pl.w = __funnelshift_r(wv[3], wv[4], sh);
          } else {
            pl = make_uint4(wv[1], wv[2], wv[3], wv[4]);
          }
          *reinterpret_cast<uint4*>(cs + Gr * (kTcChunk * 128) + b * 128 + j * 16) = pl;
          const int r = 8 * Gr + j;
          cs[kTcCanA + (b >> 2) * 512 + 16 * (r & 31) + 4 * (r >> 5) + (b & 3)] = (uint8_t)scale;
        }
        if (!ph1) {
          // B: this pair's activation planes for blocks [kb, kb + nbc) and their scales
          const uint8_t* img = a.actimg + (size_t)pp * a.img_bytes;
          const int t2 = rw * 32 + lane;  // 0..255
          if (t2 < nbc * 8) {
            const uint4 v = __ldcg(reinterpret_cast<const uint4*>(img + (size_t)kb * 128) + t2);
            *reinterpret_cast<uint4*>(cs + kTcCanA + kTcCanSFA + t2 * 16) = v;
          } else if (t2 >= 64 && t2 < 64 + nbc * 8) {
            const int q = t2 - 64, bb = q >> 3, pl = q & 7;
            const uint8_t sv = __ldcg(img + (size_t)a.nb_f * 128 + (size_t)(kb + bb) * 8 + pl);
            cs[kTcCanA + kTcCanSFA + kTcCanB + (bb >> 2) * 512 + 16 * pl + (bb & 3)] = sv;
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&full_can[cst]);
          mbar_arrive(&empty_raw[st]);
        }
      }
    }
  } else {
    // ================================================================= epilogue warps
    const int q = warp & 3;               // TMEM lane quadrant
    const int row = 32 * q + lane;        // tile row
    const int et = tid - kTcEpiWarp0 * 32;  // 0..127
    for (int sgi = 0; sgi < nseg; ++sgi) {
      const TcSeg sg = S.seg[sgi];
      const int i = sg.tile;
      const bool ph1 = i < geo.T1;
      const int db = sgi & 1;
      if (!tc_wait(&full_d[db], (sgi >> 1) & 1, abort_flag)) break;
      tc_fence_after();
      float y[NT];
      const uint32_t ta = tbase + 16 * db + ((uint32_t)(32 * q) << 16);
      if (ph1 && NT == 2) {
        uint32_t v[16];
        tmem_ld_x16(ta, v);
        tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          float s = 0.f;
#pragma unroll
          for (int pl = 0; pl < 8; ++pl) s += __uint_as_float(v[8 * t + pl]);
          y[t] = s;
        }
      } else {
        uint32_t v[8];
        tmem_ld_x8(ta, v);
        tmem_wait_ld();
        float s = 0.f;
#pragma unroll
        for (int pl = 0; pl < 8; ++pl) s += __uint_as_float(v[pl]);
        y[0] = s;
#pragma unroll
        for (int t = 1; t < NT; ++t) y[t] = 0.f;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_d[db]);
      const int ny = ph1 ? NT : 1;

      // ---- split tile: publish this segment's partial; the last CTA to arrive finishes the tile
      if (sg.nsplit > 1) {
        float* part = a.partial + ((size_t)(c * 2 + sg.my_slot) * NT) * 128;
        for (int t = 0; t < ny; ++t) __stcg(part + t * 128 + row, y[t]);
        __threadfence();
        named_sync(1, 128);
        if (et == 0) {
          const unsigned old = atomicAdd(a.cnt + i, 1u);
          S.fin = old == (unsigned)(sg.nsplit - 1);
        }
        named_sync(1, 128);
        if (!S.fin) continue;
        __threadfence();
        for (int t = 0; t < ny; ++t) {
          float s = 0.f;
          for (int g = 0; g < sg.nsplit; ++g) {
            const float* pg = a.partial + ((size_t)(sg.split_cta[g] * 2 + sg.split_slot[g]) * NT) * 128;
            s += __ldcg(pg + t * 128 + row);
          }
          y[t] = s;
        }
      }

      if (ph1) {
        // ---- phase-1 tile: rows 0..63 gate, 64..127 up of neurons 64*sl ..; activation -> planes
        const int s = i / geo.ns1, sl = i % geo.ns1;
        const int el = S.slot_expert[s] - p.expert_lo;
        for (int t = 0; t < NT; ++t) xchg[t * 128 + row] = y[t];
        named_sync(1, 128);
        if (row < 64) {
          const int n = 64 * sl + row;
          const float gb = p.gate_b ? p.gate_b[(int64_t)el * F + n] : 0.f;
          const float ub = p.up_b ? p.up_b[(int64_t)el * F + n] : 0.f;
          const int blk = n >> 5;
          for (int pp = S.slot_pair0[s]; pp < S.slot_pair0[s + 1]; ++pp) {
            const int t = S.pair_token[pp];
            const float gv = xchg[t * 128 + row] + gb, uv = xchg[t * 128 + 64 + row] + ub;
            const float av = activate(p.act_mode, gv, uv, p.alpha, p.limit);
            // planes of the 32-value block `blk` (this warp): lanes 0..15 and 16..31 pair up
            float m = fabsf(av);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            const int e = block_exp(m);
            const bool nz = m > 0.f;
            const uint32_t cd = nz ? digit_planes(av, e) : 0u;
            const uint32_t hi = __shfl_down_sync(0xffffffffu, cd, 16);
            uint8_t* img = a.actimg + (size_t)pp * a.img_bytes;
            if (lane < 16) {
#pragma unroll
              for (int pl = 0; pl < 8; ++pl) {
                const uint32_t bv = ((cd >> (4 * pl)) & 15u) | (((hi >> (4 * pl)) & 15u) << 4);
                img[(size_t)blk * 128 + pl * 16 + lane] = (uint8_t)bv;
              }
            } else if (lane < 24) {
              const int pl = lane - 16;
              img[(size_t)a.nb_f * 128 + (size_t)blk * 8 + pl] = (uint8_t)plane_scale(pl, e, nz);
            }
          }
        }
        __threadfence();
        named_sync(1, 128);
        if (et == 0) atomicAdd(a.ready + s, 1u);
      } else {
        // ---- phase-2 tile: down rows of one pair; the last pair of a row block combines it
        const int qq = i - geo.T1, pp = qq / geo.nr2, rt = qq % geo.nr2;
        const int el = S.slot_expert[S.pair_slot[pp]] - p.expert_lo;
        const int r = 128 * rt + row;
        if (r < H) {
          const float v = y[0] + (p.down_b ? p.down_b[(int64_t)el * H + r] : 0.f);
          __stcg(a.yp + (size_t)pp * H + r, v);
        }
        __threadfence();
        named_sync(1, 128);
        if (et == 0) {
          const unsigned old = atomicAdd(a.cnt2 + rt, 1u);
          S.fin = old == (unsigned)(S.npairs - 1);
        }
        named_sync(1, 128);
        if (S.fin) {
          __threadfence();
          if (r < H)
            for (int t = 0; t < T; ++t) {
              float o = 0.f;
              for (int q2 = 0; q2 < S.npairs; ++q2)
                if (S.pair_token[q2] == t) o = __fadd_rn(o, __fmul_rn(S.pair_w[q2], __ldcg(a.yp + (size_t)q2 * H + r)));
              p.out[(int64_t)t * H + r] = p.add_residual ? __fadd_rn(p.x[(int64_t)t * H + r], o) : o;
            }
        }
      }
    }
    if (et == 0) stamp(a.trace, kEvTilesEnd);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, kTcTmemCols);
  }
  if (tid == 0) stamp(a.trace, kEvEnd);
}

// ----------------------------------------------------------------------------- host side

struct TcPlan {
  size_t ws_total;
  size_t off_logits, off_partial, off_img, off_yp;
  int img_bytes, max_tiles, grid;
};

// Layers the tensor-core kernel takes: MXFP4 experts, T <= 2, H and F multiples of 64 with at
// most 16 chunks per row, 16-byte aligned expert tensors.
static bool moe_tc_eligible(const ns_moe_layer_t* p) {
  if (p->ggml_type != NS_GGML_MXFP4 || p->T > 2) return false;
  if (p->H % 64 || p->F % 64 || p->H / 32 > kTcChunk * kTcMaxSplit || p->F / 32 > kTcChunk * kTcMaxSplit) return false;
  if (p->T * p->k > kMaxPairs) return false;
  const int pairs = p->T * p->k;
  const int64_t tiles = (int64_t)pairs * (p->F / 64) + (int64_t)pairs * ((p->H + 127) / 128);
  if (tiles > kTcMaxTiles || (p->H + 127) / 128 > kTcMaxRowTiles) return false;
  return true;
}

static bool moe_tc_aligned(const ns_moe_layer_t* p) {
  auto al = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  return al(p->gate_w) && al(p->up_w) && al(p->down_w);
}

static void moe_tc_plan(const ns_moe_layer_t* p, int grid, TcPlan* t) {
  const int pairs = p->T * p->k;
  const int nb_f = p->F / 32;
  t->grid = grid;
  t->img_bytes = (int)align_up((size_t)nb_f * 128 + (size_t)nb_f * 8, 256);
  t->max_tiles = pairs * (p->F / 64) + pairs * ((p->H + 127) / 128);
  size_t off = kTcWsHeader;
  t->off_logits = off;
  off += align_up((size_t)p->T * p->n_expert * 4, 256);
  t->off_partial = off;
  off += align_up((size_t)grid * 2 * p->T * 128 * 4, 256);
  t->off_img = off;
  off += (size_t)pairs * t->img_bytes;
  t->off_yp = off;
  off += align_up((size_t)pairs * p->H * 4, 256);
  t->ws_total = off;
}

static size_t moe_tc_smem(const ns_moe_layer_t* p, MoeTcArgs* a) {
  const int nb_h = p->H / 32;
  size_t off = 0;
  a->off_raw = 0;
  off = std::max((size_t)kTcRawStages * kTcRawBytes, align_up((size_t)p->T * p->H * 4, 1024));
  off = align_up(off, 1024);
  a->off_b1 = (int)off;
  off += (size_t)p->T * nb_h * 128;
  off = align_up(off, 128);
  a->off_sfb1 = (int)off;
  a->sfb1_atom = 128 * p->T;
  off += (size_t)((nb_h + 3) / 4) * a->sfb1_atom + 512;
  off = align_up(off, 1024);
  a->off_can = (int)off;
  off += (size_t)kTcCanStages * kTcCanBytes;
  a->off_xchg = (int)off;
  off += 2 * 128 * 4;
  off = align_up(off, 64);
  a->off_bars = (int)off;
  off += 32 * 8;
  off = align_up(off, 16);
  a->off_shared = (int)off;
  off += sizeof(TcShared);
  return off;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static int get_encode_fn(EncodeTiledFn* out) {
  static EncodeTiledFn fn = nullptr;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !ptr)
      return fail(NS_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  *out = fn;
  return NS_OK;
}

// Tensor map over `rows` GGUF rows of `rb` bytes viewed as (rows/8) groups of 8*rb bytes.
static int make_row_group_map(CUtensorMap* m, const uint8_t* base, int64_t rows, int rb) {
  EncodeTiledFn fn;
  int st = get_encode_fn(&fn);
  if (st) return st;
  const cuuint64_t dims[2] = {(cuuint64_t)8 * rb, (cuuint64_t)(rows / 8)};
  const cuuint64_t strides[1] = {(cuuint64_t)8 * rb};
  const cuuint32_t box[2] = {(cuuint32_t)kTcBoxW, 8};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NS_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return NS_OK;
}

template <int NT>
static int launch_moe_tc(const MoeTcArgs& a, int grid, size_t smem, cudaStream_t stream) {
  auto kern = moe_tc_kernel<NT>;
  NS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int per_sm = 0;
  NS_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kTcThreads, smem));
  if (per_sm < 1) return fail(NS_ERR_UNSUPPORTED, "ns_moe_decode_layer: tensor-core kernel does not fit on an SM");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  NS_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a));
  return NS_OK;
}

static int moe_tc_launch(const ns_moe_layer_t* p, const TcPlan& tp, uint8_t* ws, cudaStream_t s) {
  MoeTcArgs a;
  memset(&a, 0, sizeof a);
  a.p = *p;
  a.rb_h = (int)row_bytes_of(p->ggml_type, p->H);
  a.rb_f = (int)row_bytes_of(p->ggml_type, p->F);
  a.nb_h = p->H / 32;
  a.nb_f = p->F / 32;
  const int n_local = p->expert_hi - p->expert_lo;
  int st = make_row_group_map(&a.tm_gate, p->gate_w, (int64_t)n_local * p->F, a.rb_h);
  if (!st) st = make_row_group_map(&a.tm_up, p->up_w, (int64_t)n_local * p->F, a.rb_h);
  if (!st) st = make_row_group_map(&a.tm_down, p->down_w, (int64_t)n_local * p->H, a.rb_f);
  if (st) return st;
  a.bar = reinterpret_cast<unsigned long long*>(ws);
  a.cnt = reinterpret_cast<unsigned*>(ws + kTcOffCnt);
  a.ready = reinterpret_cast<unsigned*>(ws + kTcOffReady);
  a.cnt2 = reinterpret_cast<unsigned*>(ws + kTcOffCnt2);
  a.logits = reinterpret_cast<float*>(ws + tp.off_logits);
  a.partial = reinterpret_cast<float*>(ws + tp.off_partial);
  a.actimg = ws + tp.off_img;
  a.yp = reinterpret_cast<float*>(ws + tp.off_yp);
  a.img_bytes = tp.img_bytes;
  a.zero_tiles = tp.max_tiles;
  a.trace = g_trace_buf[trace_slot()];
  const size_t smem = moe_tc_smem(p, &a);
  if (smem > (size_t)kTcSmemBudget)
    return fail(NS_ERR_UNSUPPORTED, "ns_moe_decode_layer: tensor-core layout needs %zu bytes of shared memory", smem);
  if (tp.grid > 1024) return fail(NS_ERR_UNSUPPORTED, "ns_moe_decode_layer: more than 1024 SMs");
  return p->T == 1 ? launch_moe_tc<1>(a, tp.grid, smem, s) : launch_moe_tc<2>(a, tp.grid, smem, s);
}

}  // namespace ns
