// MoE decode step on device: router (ns_moe_route) and the fused layer
// (ns_moe_decode_layer).
//
// The fused layer is ONE cooperative launch of one CTA per SM:
//   1. every CTA: h = RMSNorm(x) into shared memory (redundant, H floats);
//   2. router logits, one expert per CTA (CTA c: experts c, c+G, ...) -> workspace;
//   3. grid barrier; every CTA re-derives top-k + weights from the logits and
//      builds the routed-expert slots (ascending expert id, as the reference
//      walks torch.unique(ids)) and its own tile list;
//   4. phase 1: the (slot, neuron) space is split evenly over CTAs; a tile is
//      up to 12 neurons of one slot (their gate and up rows);
//   5. grid barrier; phase 2: output rows are split evenly over CTAs; a tile is
//      this CTA's rows (up to 24) of one slot's down matrix, slots in
//      ascending expert order, accumulating w * (down.a + b) per row in the
//      reference's order; then the residual is added.
//
// Inside a CTA, one producer warp streams tiles (1-D bulk copies on the TMA
// engine) through a ring of shared-memory stages guarded by full/empty
// mbarriers, so weight bytes keep flowing across both grid barriers.  Twelve
// consumer warps split each tile as 3 row-groups x 4 K-chunks; every
// (group, chunk) partial lands in shared memory and the group's four warps
// reduce them in a fixed order (results are deterministic).  MXFP4 tiles run
// on the tensor cores (mma_mxfp4.cuh); Q8_0 and Q4_K launches of one or two
// tokens run dp4a against int8 digit planes of the activations (unit_int8);
// the other K-quant cases use the CUDA-core group decoders (qdot.cuh).  Every
// device wait is bounded.
#include <mutex>

#include "mma_mxfp4.cuh"
#include "qdot.cuh"

namespace ns {

constexpr int kMaxPairs = NS_MAX_TOKENS * NS_MAX_TOPK;  // (slot, token) pairs
constexpr int kWsHeader = 1024;  // workspace: barrier counter at 0, activation maxima at 64
constexpr int kMaxTiles = 300;  // Qwen3-235B batch 8 (T=8 x k=8 Q4_K, 2 stages of 8-neuron tiles) needs 277
constexpr int kMoeSmemBudget = 225 * 1024;

// ----------------------------------------------------------------------------- routing helpers

// Top-k of v[0..E) by (value desc, index asc), one warp.  Writes ids/vals to smem arrays.
__device__ void warp_topk(const float* v, int E, int k, int* ids, float* vals, int lane) {
  // lane holds experts lane + 32*i (i < 16); bit i of `taken` marks one already chosen
  uint32_t taken = 0u;
  float mine[NS_MAX_EXPERTS / 32];
#pragma unroll
  for (int i = 0; i < NS_MAX_EXPERTS / 32; ++i) {
    const int e = lane + 32 * i;
    mine[i] = e < E ? v[e] : 0.f;
  }
  for (int j = 0; j < k; ++j) {
    float best = -INFINITY;
    int bi = 0x7FFFFFFF;
#pragma unroll
    for (int i = 0; i < NS_MAX_EXPERTS / 32; ++i) {
      const int e = lane + 32 * i;
      if (e >= E || ((taken >> i) & 1u)) continue;
      const float x = mine[i];
      if (bi == 0x7FFFFFFF || x > best || (x == best && e < bi)) {
        best = x;
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ob = __shfl_xor_sync(0xffffffffu, best, o);
      int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (oi != 0x7FFFFFFF && (bi == 0x7FFFFFFF || ob > best || (ob == best && oi < bi))) {
        best = ob;
        bi = oi;
      }
    }
    if (bi == 0x7FFFFFFF) bi = 0;  // E < k cannot happen (validated on the host)
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    if (lane == 0) {
      ids[j] = bi;
      vals[j] = best;
    }
  }
}

// Route one token from its logits (one warp).  GPT-OSS: top-k of logits then
// softmax over the k.  Qwen3: softmax over all, top-k, renormalise.
// `scratch` holds E floats of shared memory for the Qwen probabilities.
__device__ void warp_route(const float* logits, int E, int k, int mode, int* ids, float* w, float* scratch,
                           int lane) {
  if (mode == NS_ROUTE_TOPK_SOFTMAX) {
    warp_topk(logits, E, k, ids, w, lane);
    __syncwarp();
    if (lane == 0) {
      float m = w[0];
      float s = 0.f;
      for (int j = 0; j < k; ++j) {
        w[j] = expf(w[j] - m);
        s += w[j];
      }
      for (int j = 0; j < k; ++j) w[j] = w[j] / s;
    }
  } else {
    float m = -INFINITY;
    for (int e = lane; e < E; e += 32) m = fmaxf(m, logits[e]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = 0.f;
    for (int e = lane; e < E; e += 32) {
      float p = expf(logits[e] - m);
      scratch[e] = p;
      s += p;
    }
    s = warp_sum(s);
    for (int e = lane; e < E; e += 32) scratch[e] = scratch[e] / s;
    __syncwarp();
    warp_topk(scratch, E, k, ids, w, lane);
    __syncwarp();
    if (lane == 0) {
      float t = 0.f;
      for (int j = 0; j < k; ++j) t += w[j];
      for (int j = 0; j < k; ++j) w[j] = w[j] / t;
    }
  }
  __syncwarp();
}

// ----------------------------------------------------------------------------- standalone router

// logits[t][e] = h[t] . W[e] (+ b[e]); one warp per (t, e).
__global__ void route_logits_kernel(const void* h, int h_dtype, int T, int H, const void* w, int w_dtype,
                                    const float* b, int E, float* logits) {
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (gw >= T * E) return;
  const int t = gw / E, e = gw - t * E;
  float s = 0.f;
  for (int i = lane; i < H; i += 32)
    s = fmaf(load_float(h, h_dtype, (int64_t)t * H + i), load_float(w, w_dtype, (int64_t)e * H + i), s);
  s = warp_sum(s);
  if (lane == 0) logits[(int64_t)t * E + e] = b ? s + b[e] : s;
}

// One warp per token.
__global__ void route_select_kernel(const float* logits, int T, int E, int k, int mode, int32_t* ids,
                                    float* weights) {
  extern __shared__ float route_smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t = blockIdx.x * (blockDim.x >> 5) + warp;
  float* scratch = route_smem + warp * (NS_MAX_EXPERTS + 2 * NS_MAX_TOPK);
  int* sid = reinterpret_cast<int*>(scratch + NS_MAX_EXPERTS);
  float* sw = scratch + NS_MAX_EXPERTS + NS_MAX_TOPK;
  if (t >= T) return;
  warp_route(logits + (int64_t)t * E, E, k, mode, sid, sw, scratch, lane);
  if (lane < k) {
    ids[t * k + lane] = sid[lane];
    weights[t * k + lane] = sw[lane];
  }
}

// ----------------------------------------------------------------------------- fused layer

constexpr int kComputeWarps = 12;
constexpr int kGroups = 3;          // row-groups of 8 weight rows per tile
constexpr int kKChunks = 4;         // K-chunks per tile (kGroups * kKChunks = kComputeWarps)
constexpr int kTileCols = 24;       // weight rows per tile
constexpr int kMoeThreads = (kComputeWarps + 1) * 32;
constexpr int kComputeThreads = kComputeWarps * 32;
constexpr int kProducerWarp = kComputeWarps;
constexpr int kMaxStages = 4;
constexpr int kRedFloats = kKChunks * kTileCols * 16;  // one parity of the partial-sum buffer

struct MoeArgs {
  ns_moe_layer_t p;
  int rb_h, rb_f;          // bytes of a gate/up row (K=H) and of a down row (K=F)
  int nb_h, nb_f;          // 32-element blocks per row
  int n_local;
  const uint8_t* gate_end;
  const uint8_t* up_end;
  const uint8_t* down_end;
  float* logits;           // workspace: T x E
  float* act;              // workspace: pairs x F
  unsigned* amax;          // workspace: max |activation| bits per pair (kMaxPairs)
  unsigned long long* bar;
  int stages, stage_bytes, half;
  int tn;                  // phase-1 neurons per tile (<= 12)
  int tr;                  // phase-2 rows per tile (<= 24)
  int rows_cta_max;        // phase-2 output rows per CTA, upper bound
  int sc_stride;           // floats of each warp's scale buffer
  int act_global;          // CUDA-core path: phase 2 reads the activation rows from the workspace (L2)
                           // instead of a shared-memory copy (pairs x F floats beyond shared memory)
  // shared-memory layout (byte offsets)
  int off_oacc, off_red, off_sc, off_stages, off_bars, off_shared, off_bias;
  unsigned long long* trace;  // per-CTA phase stamps, or nullptr
};

// Phase stamps (event ids of ns_moe_set_trace)
enum { kEvStart = 0, kEvNorm, kEvRouter, kEvBarrier1, kEvRoute, kEvImages, kEvFirstTile, kEvPhase1End,
       kEvBarrier2, kEvPhase2Images, kEvTilesEnd, kEvEnd, kEvProducerFirst, kEvProducerLast, kEvLogits,
       kEvTopk };

__device__ __forceinline__ void stamp(unsigned long long* tr, int ev) {
  if (tr) tr[blockIdx.x * NS_TRACE_EVENTS + ev] = globaltimer_ns();
}

struct Tile {
  short phase;  // 1 or 2
  short slot;
  int r0, r1;   // neuron range (phase 1) or output-row range (phase 2)
};

struct MoeShared {
  int ids[NS_MAX_TOKENS][NS_MAX_TOPK];
  float w[NS_MAX_TOKENS][NS_MAX_TOPK];
  int nslots, npairs, ntiles, n1_tiles;
  int slot_expert[kMaxPairs];
  int slot_pair0[kMaxPairs + 1];
  int pair_token[kMaxPairs];
  float pair_w[kMaxPairs];
  float fac_tok[NS_MAX_TOKENS];   // 2^(1-sigma) of each token's h image (1 on the CUDA-core path)
  float fac_pair[kMaxPairs];      // same for each activation image
  int sig_tok[NS_MAX_TOKENS];
  int sig_pair[kMaxPairs];
  int ok;
  unsigned long long bar_target;
  float rscale[NS_MAX_TOKENS];
  float topv[NS_MAX_TOKENS][NS_MAX_TOPK];
  float red[kComputeWarps + 1][NS_MAX_TOKENS];
  float red2[kComputeWarps + 1][NS_MAX_TOKENS];
  Tile tiles[kMaxTiles];
  __align__(16) float scratch[NS_MAX_EXPERTS];
};

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Grid-wide barrier on a monotonically increasing 64-bit counter: barrier
// instance n completes when the counter reaches (n+1)*G.  Bounded wait.
// Called by thread 0 only; the caller synchronises its CTA around it.
__device__ int grid_barrier_thread0(unsigned long long* bar, unsigned G) {
  __threadfence();
  unsigned long long old = atomicAdd(bar, 1ull);
  unsigned long long target = (old / G + 1ull) * G;
  uint64_t t0 = globaltimer_ns();
  while (ld_acquire_u64(bar) < target) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      raise_device_error(NS_DEVERR_GRID_WAIT);
      return 0;
    }
    __nanosleep(32);
  }
  return 1;
}

__device__ __forceinline__ float activate(int mode, float g, float u, float alpha, float limit) {
  if (mode == NS_ACT_CLAMPED_SWIGLU) {
    // neurostream/model/gpt_oss.py:61-70, operation for operation
    g = fminf(g, limit);
    u = fminf(fmaxf(u, -limit), limit);
    float sg = 1.0f / (1.0f + expf(-__fmul_rn(g, alpha)));
    return __fmul_rn(__fadd_rn(u, 1.0f), __fmul_rn(g, sg));
  }
  float sg = 1.0f / (1.0f + expf(-g));
  return __fmul_rn(__fmul_rn(g, sg), u);
}

// Weight-row address of tile column c (0..23) in the staged tile.
// Phase 1: group gi = c/8 holds neurons 4gi..4gi+3; column 8gi + 2j is the
// gate row of neuron 4gi+j and 8gi + 2j + 1 its up row.  Phase 2: column c is
// tile row c.  Columns past the tile's rows point at its last row.
__device__ __forceinline__ const uint8_t* tile_row(int phase, int c, const uint8_t* s0base, const uint8_t* s1base,
                                                   int nvalid, int rb) {
  if (phase == 1) {
    int n = (c >> 3) * 4 + ((c & 7) >> 1);
    n = min(n, nvalid - 1);
    return ((c & 1) ? s1base : s0base) + (int64_t)n * rb;
  }
  return s0base + (int64_t)min(c, nvalid - 1) * rb;
}

// The tile's spans (bulk-copy sources) and their buffers.
struct TileSpans {
  Span s0, s1;
  const uint8_t *b0, *e0, *b1, *e1;
};

__device__ __forceinline__ TileSpans tile_spans(const MoeArgs& a, const MoeShared& S, int i) {
  const ns_moe_layer_t& p = a.p;
  const Tile tl = S.tiles[i];
  const int el = S.slot_expert[tl.slot] - p.expert_lo;
  TileSpans t;
  if (tl.phase == 1) {
    const int64_t row0 = (int64_t)el * p.F + tl.r0, row1 = (int64_t)el * p.F + tl.r1;
    t.s0 = Span{p.gate_w + row0 * a.rb_h, p.gate_w + row1 * a.rb_h};
    t.s1 = Span{p.up_w + row0 * a.rb_h, p.up_w + row1 * a.rb_h};
    t.b0 = p.gate_w;
    t.e0 = a.gate_end;
    t.b1 = p.up_w;
    t.e1 = a.up_end;
  } else {
    const int64_t row0 = (int64_t)el * p.H + tl.r0, row1 = (int64_t)el * p.H + tl.r1;
    t.s0 = Span{p.down_w + row0 * a.rb_f, p.down_w + row1 * a.rb_f};
    t.s1 = Span{nullptr, nullptr};
    t.b0 = p.down_w;
    t.e0 = a.down_end;
    t.b1 = t.e1 = nullptr;
  }
  return t;
}

// One (group, K-chunk) unit of a tile on the CUDA-core path: writes
// red[kc][col][2i] = partial dot of tile column col with token i and
// red[kc][col][2i+1] = 0.
template <int FMT, int NT>
__device__ __forceinline__ void unit_cuda_core(int phase, int gi, int kc, const uint8_t* s0base,
                                               const uint8_t* s1base, int nvalid, int rb, int ngroups,
                                               const float* x, int64_t xs, const int (&tok)[NT], int nt,
                                               float* red, int lane) {
  using G = QGroup<FMT>;
  const int g0 = (ngroups * kc) / kKChunks, g1 = (ngroups * (kc + 1)) / kKChunks;
#pragma unroll 1
  for (int hf = 0; hf < 2; ++hf) {
    const uint8_t* rs[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) rs[r] = tile_row(phase, 8 * gi + 4 * hf + r, s0base, s1base, nvalid, rb);
    float part[4][NT];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int t = 0; t < NT; ++t) part[r][t] = 0.f;
    for (int g = g0 + lane; g < g1; g += 32) {
      G qg[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) qg[r].load(rs[r], g);
      float pt[4][NT][G::kParts];
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
          for (int pp = 0; pp < G::kParts; ++pp) pt[r][t][pp] = 0.f;
      float xsum[NT];
#pragma unroll
      for (int t = 0; t < NT; ++t) xsum[t] = 0.f;
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        float xv[NT][8];
        G::template load_x<NT>(x, xs, tok, nt, g, s, xv);
        if (FMT == NS_GGML_Q4_K) {
#pragma unroll
          for (int t = 0; t < NT; ++t)
            if (t < nt)
              xsum[t] += ((xv[t][0] + xv[t][1]) + (xv[t][2] + xv[t][3])) + ((xv[t][4] + xv[t][5]) + (xv[t][6] + xv[t][7]));
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) qg[r].template fma<NT>(s, xv, nt, pt[r]);
      }
#pragma unroll
      for (int r = 0; r < 4; ++r) qg[r].template finish<NT>(pt[r], xsum, nt, part[r]);
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        float v = warp_sum(part[r][t]);
        if (lane == 0 && t < nt) {
          const int col = 8 * gi + 4 * hf + r;
          red[(kc * kTileCols + col) * 16 + 2 * t] = v;
          red[(kc * kTileCols + col) * 16 + 2 * t + 1] = 0.f;
        }
      }
    }
  }
}

// Layers whose Q8_0 / Q4_K experts run on dp4a against int8 activation planes (one or two tokens:
// the planes of h and of every pair's activation row fit the shared-memory region).
__host__ __device__ constexpr bool moe_int8_path(int fmt, int nt) {
  return (fmt == NS_GGML_Q4_K || fmt == NS_GGML_Q8_0) && nt <= 2;
}

// The same unit for Q8_0 and Q4_K on dp4a: the activations are int8 digit planes (kXQG bytes per
// group, token slot t's group g at xq + t*xqs + g*kXQG, its scale and sum at xsc / xsum[t*ngroups
// + g]); each group's dot product is three exact integer dp4a chains per weight word, combined in
// fp32 and scaled once (the fused GEMV's integer path).  rows16: the tile's rows start on 16-byte
// boundaries (Q4_K superblocks then load as three vectors).
template <int FMT, int NT>
__device__ __forceinline__ void unit_int8(int phase, int gi, int kc, const uint8_t* s0base, const uint8_t* s1base,
                                          int nvalid, int rb, int ngroups, const uint8_t* xq, int xqs,
                                          const float* xsc, const float* xsum, const int (&tok)[NT], int nt,
                                          float* red, int lane, bool rows16) {
  const int g0 = (ngroups * kc) / kKChunks, g1 = (ngroups * (kc + 1)) / kKChunks;
  // a chunk of at most 16 groups (short rows, e.g. the down rows of narrow experts): the two
  // 4-row halves run at once on the two 16-lane halves of the warp instead of one after the other
  const bool both = g1 - g0 <= 16;
  const int step = both ? 16 : 32, ln = both ? (lane & 15) : lane;
#pragma unroll 1
  for (int pass = 0; pass < (both ? 1 : 2); ++pass) {
    const int hf = both ? (lane >> 4) : pass;
    const uint8_t* rs[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) rs[r] = tile_row(phase, 8 * gi + 4 * hf + r, s0base, s1base, nvalid, rb);
    float acc[4][NT];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;
    for (int g = g0 + ln; g < g1; g += step) {
      uint32_t q[4][8];
      float da[4], db[4];  // Q8_0: d, 0; Q4_K: d*sc, dmin*mn
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        if (FMT == NS_GGML_Q8_0) {
          uint32_t w[9];
          lds_words_unaligned<9>(rs[r] + 34 * g, w);
          da[r] = f16_bits_to_float(w[0]);
          db[r] = 0.f;
#pragma unroll
          for (int i = 0; i < 8; ++i) q[r][i] = __funnelshift_r(w[i], w[i + 1], 16);  // signed int8 x 4
        } else {
          QGroup<NS_GGML_Q4_K> qg;
          if (rows16)
            qg.load_aligned(rs[r], g);
          else
            qg.load(rs[r], g);
          da[r] = qg.dsc;
          db[r] = qg.mmn;
#pragma unroll
          for (int i = 0; i < 8; ++i) q[r][i] = qg.q[i];  // 0..15 x 4
        }
      }
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        if (t >= nt) continue;
        const uint4* xp = reinterpret_cast<const uint4*>(xq + (size_t)tok[t] * xqs + (size_t)g * kXQG);
        uint32_t xw[3][8];
#pragma unroll
        for (int pl = 0; pl < 3; ++pl) {
          const uint4 lo = xp[2 * pl], hi = xp[2 * pl + 1];
          xw[pl][0] = lo.x; xw[pl][1] = lo.y; xw[pl][2] = lo.z; xw[pl][3] = lo.w;
          xw[pl][4] = hi.x; xw[pl][5] = hi.y; xw[pl][6] = hi.z; xw[pl][7] = hi.w;
        }
        const float sc = xsc[tok[t] * ngroups + g], sm = xsum[tok[t] * ngroups + g];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          int s0 = 0, s1 = 0, s2 = 0;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            s0 = __dp4a((int)q[r][i], (int)xw[0][i], s0);
            s1 = __dp4a((int)q[r][i], (int)xw[1][i], s1);
            s2 = __dp4a((int)q[r][i], (int)xw[2][i], s2);
          }
          const float f = fmaf((float)s2, 65536.f, fmaf((float)s1, 256.f, (float)s0)) * sc;
          acc[r][t] = fmaf(f, da[r], FMT == NS_GGML_Q4_K ? fmaf(-db[r], sm, acc[r][t]) : acc[r][t]);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        float v = acc[r][t];  // sum over the lanes of this half (or of the warp)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
          if (o < step) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (ln == 0 && t < nt) {
          const int col = 8 * gi + 4 * hf + r;
          red[(kc * kTileCols + col) * 16 + 2 * t] = v;
          red[(kc * kTileCols + col) * 16 + 2 * t + 1] = 0.f;
        }
      }
    }
  }
}

template <int FMT, int NT>
__global__ void __launch_bounds__(kMoeThreads, 1) moe_layer_kernel(MoeArgs a) {
  constexpr bool kMma = (FMT == NS_GGML_MXFP4);
  constexpr bool kInt = moe_int8_path(FMT, NT);  // dp4a on int8 activation planes
  extern __shared__ __align__(128) uint8_t smem[];
  const ns_moe_layer_t& p = a.p;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) l2_prefetch_share(a.p.l2, blockIdx.x, gridDim.x);  // the next kernels' weights (hint)
  const int G = gridDim.x, c = blockIdx.x;
  const int T = p.T, H = p.H, F = p.F, E = p.n_expert, k = p.k;

  float* region = reinterpret_cast<float*>(smem);
  float* o_acc = reinterpret_cast<float*>(smem + a.off_oacc);
  float* red_base = reinterpret_cast<float*>(smem + a.off_red);
  float* sc_base = reinterpret_cast<float*>(smem + a.off_sc);
  uint8_t* stages = smem + a.off_stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bars);
  uint64_t* empty = full + kMaxStages;
  float* stage_bias = reinterpret_cast<float*>(smem + a.off_bias);  // kTileCols floats per stage
  MoeShared& S = *reinterpret_cast<MoeShared*>(smem + a.off_shared);

  if (tid == 0) {
    stamp(a.trace, kEvStart);
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], 2);  // producer: bulk-copy arm + bias/ragged bytes written
      mbar_init(&empty[s], kComputeWarps);
    }
    fence_mbar_init();
  }

  if (c == 0 && tid < kMaxPairs) a.amax[tid] = 0u;  // activation maxima of this launch (phase 1 -> 2)

  // ---- 1+2. one pass over the layer input: raw x into shared memory, sum of
  // squares for RMSNorm, and this CTA's router logit in the same loop.  The
  // norm is a per-token scalar r times the weight w, so
  //   logit = sum_i (x_i r w_i) W_ci = r * sum_i (x_i w_i) W_ci.
  float* h = region;
  const bool own_expert = c < E;
  for (int t = 0; t < T; ++t) {
    float ss = 0.f, dot = 0.f;
    for (int i0 = tid; i0 < H; i0 += 8 * kMoeThreads) {  // 8 elements' loads in flight, then summed in order
      float xv[8], wv[8], rv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + u * kMoeThreads;
        xv[u] = i < H ? p.x[(int64_t)t * H + i] : 0.f;
        wv[u] = i < H && p.norm_w ? p.norm_w[i] : 1.0f;
      }
      load_floats<8>(p.router_w, p.router_dtype, [&](int u) -> int64_t {
        const int i = i0 + u * kMoeThreads;
        return i < H && own_expert ? (int64_t)c * H + i : -1;
      }, rv);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + u * kMoeThreads;
        if (i < H) {
          h[t * H + i] = xv[u];
          ss = fmaf(xv[u], xv[u], ss);
          dot = fmaf(xv[u] * wv[u], rv[u], dot);
        }
      }
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
    for (int w = 0; w <= kComputeWarps; ++w) {
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
      for (int i = tid; i < H; i += kMoeThreads) h[t * H + i] = __fmul_rn(__fmul_rn(h[t * H + i], r), p.norm_w[i]);
    }
  __syncthreads();
  if (tid == 0) stamp(a.trace, kEvNorm);

  // more experts than CTAs: the rest of this CTA's router rows from h
  for (int e = c + G; e < E; e += G) {
    float sacc[NS_MAX_TOKENS];
#pragma unroll
    for (int t = 0; t < NS_MAX_TOKENS; ++t) sacc[t] = 0.f;
    for (int i = tid; i < H; i += kMoeThreads) {
      const float wv = load_float(p.router_w, p.router_dtype, (int64_t)e * H + i);
#pragma unroll
      for (int t = 0; t < NS_MAX_TOKENS; ++t)
        if (t < T) sacc[t] = fmaf(h[t * H + i], wv, sacc[t]);
    }
#pragma unroll
    for (int t = 0; t < NS_MAX_TOKENS; ++t)
      if (t < T) {
        const float v = warp_sum(sacc[t]);
        if (lane == 0) S.red[warp][t] = v;
      }
    __syncthreads();
    if (tid < T) {
      float v = 0.f;
      for (int w = 0; w <= kComputeWarps; ++w) v += S.red[w][tid];
      a.logits[(int64_t)tid * E + e] = v + (p.router_b ? p.router_b[e] : 0.f);
    }
    __syncthreads();
  }

  // ---- 3. split-phase grid barrier: arrive now, build the h images, wait later
  if (tid == 0) {
    stamp(a.trace, kEvRouter);
    __threadfence();
    const unsigned long long old = atomicAdd(a.bar, 1ull);
    S.bar_target = (old / (unsigned)G + 1ull) * (unsigned)G;
  }
  uint4* ximg = reinterpret_cast<uint4*>(region + ((T * H + 31) / 32) * 32);
  if (kMma) {
    for (int t = 0; t < T; ++t) {
      float m = 0.f;
      for (int i = tid; i < H; i += kMoeThreads) m = fmaxf(m, fabsf(h[t * H + i]));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (lane == 0) S.red[warp][t] = m;
    }
    __syncthreads();
    if (tid < T) {
      float m = 0.f;
      for (int w = 0; w <= kComputeWarps; ++w) m = fmaxf(m, S.red[w][tid]);
      const int sg = xsplit_sigma(m);
      S.sig_tok[tid] = sg;
      S.fac_tok[tid] = ldexpf(1.0f, 1 - sg);
    }
    __syncthreads();
    for (int t = 0; t < T; ++t)
      build_xfrag(h + t * H, a.nb_h, S.sig_tok[t], ximg + t * xfrag_vec_u4(a.nb_h), tid, kMoeThreads);
  } else {
    if (tid < T) S.fac_tok[tid] = 1.0f;
    if (kInt && tid >= 32) {
      // h of every token as int8 digit planes, one thread per (token, group); warp 0 stays free, so
      // thread 0 polls the grid barrier as soon as it completes
      uint8_t* xq = reinterpret_cast<uint8_t*>(ximg);
      float* xsc = reinterpret_cast<float*>(xq + (size_t)T * a.nb_h * kXQG);
      float* xsm = xsc + T * a.nb_h;
      for (int it = tid - 32; it < T * a.nb_h; it += kMoeThreads - 32) {
        const int t = it / a.nb_h, g = it - t * a.nb_h;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = h[t * H + 32 * g + j];
        group_planes_i8(v, xq + (size_t)it * kXQG, &xsc[it], &xsm[it]);
      }
    }
  }
  for (int i = tid; i < T * a.rows_cta_max; i += kMoeThreads) o_acc[i] = 0.f;
  if (tid == 0) {
    S.ok = 1;
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_u64(a.bar) < S.bar_target) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        raise_device_error(NS_DEVERR_GRID_WAIT);
        S.ok = 0;
        break;
      }
      __nanosleep(32);
    }
    stamp(a.trace, kEvBarrier1);
  }
  __syncthreads();

  // ---- 4. routing: every thread ranks one expert against all (value desc,
  // index asc -- the order torch.topk returns), so the k winners are found in
  // one parallel pass instead of k sequential arg-max rounds.
  float* sc_e = S.scratch;  // scores of the current token
  for (int t = 0; t < T; ++t) {
    const float lg = tid < E ? __ldcg(a.logits + (int64_t)t * E + tid) : -INFINITY;
    float score = lg;
    if (p.route_mode == NS_ROUTE_SOFTMAX_TOPK_NORM) {
      // softmax over all experts first (neurostream/moe/router.py:64-65)
      float m = lg;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (lane == 0) S.red[warp][0] = m;
      __syncthreads();
      m = S.red[0][0];
      for (int w = 1; w <= kComputeWarps; ++w) m = fmaxf(m, S.red[w][0]);
      const float ex = tid < E ? expf(lg - m) : 0.f;
      float sum = warp_sum(ex);
      __syncthreads();
      if (lane == 0) S.red[warp][0] = sum;
      __syncthreads();
      sum = 0.f;
      for (int w = 0; w <= kComputeWarps; ++w) sum += S.red[w][0];
      score = ex / sum;
    }
    if (tid < E) sc_e[tid] = score;
    __syncthreads();
    if (tid < E) {
      int rank = 0;
      int e2 = 0;
      for (; e2 + 4 <= E; e2 += 4) {
        const float4 v4 = *reinterpret_cast<const float4*>(sc_e + e2);
        rank += (v4.x > score || (v4.x == score && e2 < tid));
        rank += (v4.y > score || (v4.y == score && e2 + 1 < tid));
        rank += (v4.z > score || (v4.z == score && e2 + 2 < tid));
        rank += (v4.w > score || (v4.w == score && e2 + 3 < tid));
      }
      for (; e2 < E; ++e2) rank += (sc_e[e2] > score || (sc_e[e2] == score && e2 < tid));
      if (rank < k) {
        S.ids[t][rank] = tid;
        S.topv[t][rank] = score;
      }
    }
    __syncthreads();
    if (warp == 0) {
      const float v = lane < k ? S.topv[t][lane] : 0.f;
      float wgt;
      if (p.route_mode == NS_ROUTE_TOPK_SOFTMAX) {
        // softmax over the k (neurostream/model/gpt_oss.py:119-120)
        const float m = S.topv[t][0];
        const float ex = lane < k ? expf(v - m) : 0.f;
        wgt = ex / warp_sum(ex);
      } else {
        wgt = v / warp_sum(v);  // renormalise the top-k probabilities (router.py:66-68)
      }
      if (lane < k) S.w[t][lane] = wgt;
    }
    __syncthreads();
  }
  if (tid == 0) stamp(a.trace, kEvTopk);

  // ---- 5. slots (distinct local experts, ascending) and this CTA's tiles
  if (warp == 0) {
    if (T == 1) {
      const int e = lane < k ? S.ids[0][lane] : 0x7FFFFFFF;
      const bool local = lane < k && e >= p.expert_lo && e < p.expert_hi;
      int rank = 0, n = 0;
      for (int j = 0; j < k; ++j) {
        const int ej = __shfl_sync(0xffffffffu, e, j);
        const bool lj = ej >= p.expert_lo && ej < p.expert_hi;
        rank += lj && ej < e;
        n += lj;
      }
      if (local) {
        S.slot_expert[rank] = e;
        S.slot_pair0[rank] = rank;
        S.pair_token[rank] = 0;
        S.pair_w[rank] = S.w[0][lane];
      }
      if (lane == 0) {
        S.slot_pair0[n] = n;
        S.nslots = n;
        S.npairs = n;
      }
    } else {
      // Lane l owns experts [32l, 32l+32) as a bitmap; a scan of the popcounts places them.
      uint32_t bits = 0u;
      for (int t = 0; t < T; ++t)
        for (int j = 0; j < k; ++j) {
          const int e = S.ids[t][j];
          if (e >= p.expert_lo && e < p.expert_hi && (e >> 5) == lane) bits |= 1u << (e & 31);
        }
      const int cnt = __popc(bits);
      int incl = cnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      const int n = __shfl_sync(0xffffffffu, incl, 31);
      {
        int pos = incl - cnt;
        for (uint32_t b = bits; b; b &= b - 1) S.slot_expert[pos++] = 32 * lane + __ffs(b) - 1;
      }
      __syncwarp();
      int base = 0;
      for (int j0 = 0; j0 < n; j0 += 32) {
        const int j = j0 + lane;
        int cj = 0;
        if (j < n)
          for (int t = 0; t < T; ++t)
            for (int q2 = 0; q2 < k; ++q2) cj += S.ids[t][q2] == S.slot_expert[j];
        int inc = cj;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int v = __shfl_up_sync(0xffffffffu, inc, o);
          if (lane >= o) inc += v;
        }
        if (j < n) {
          int pp = base + inc - cj;
          S.slot_pair0[j] = pp;
          for (int t = 0; t < T; ++t)
            for (int q2 = 0; q2 < k; ++q2)
              if (S.ids[t][q2] == S.slot_expert[j]) {
                S.pair_token[pp] = t;
                S.pair_w[pp] = S.w[t][q2];
                ++pp;
              }
        }
        base += __shfl_sync(0xffffffffu, inc, 31);
      }
      if (lane == 0) {
        S.slot_pair0[n] = base;
        S.nslots = n;
        S.npairs = base;
      }
    }
    __syncwarp();
    if (lane == 0) {
      const int n = S.nslots;
      int nt = 0;
      const int N1 = n * F;  // <= NS_MAX_TOKENS * NS_MAX_TOPK * F: int32 is enough
      int pos = N1 * c / G;
      const int end1 = N1 * (c + 1) / G;
      int j = pos / F, n0 = pos - j * F;
      while (pos < end1 && nt < kMaxTiles) {
        const int lim = min(min(n0 + a.tn, F), n0 + (end1 - pos));
        S.tiles[nt++] = Tile{1, (short)j, n0, lim};
        pos += lim - n0;
        n0 = lim;
        if (n0 == F) {
          n0 = 0;
          ++j;
        }
      }
      S.n1_tiles = nt;
      const int ra = H * c / G, rb = H * (c + 1) / G;
      for (int r0 = ra; r0 < rb; r0 += a.tr)
        for (int jj = 0; jj < n && nt < kMaxTiles; ++jj) S.tiles[nt++] = Tile{2, (short)jj, r0, min(rb, r0 + a.tr)};
      S.ntiles = nt;
      stamp(a.trace, kEvRoute);
    }
    if (c == 0)
      for (int i = lane; i < T * k; i += 32) {
        if (p.ids) p.ids[i] = S.ids[i / k][i % k];
        if (p.weights) p.weights[i] = S.w[i / k][i % k];
      }
  }
  __syncthreads();
  if (tid == 0) stamp(a.trace, kEvImages);

  const int ntiles = S.ntiles, n1_tiles = S.n1_tiles;
  const int ra = (int)((int64_t)H * c / G);

  // ================================================================= producer warp
  if (warp == kProducerWarp) {
    for (int i = 0; i < ntiles; ++i) {
      const int st = i % a.stages;
      if (i >= a.stages) {
        if (lane == 0) mbar_wait_bounded(&empty[st], (uint32_t)(((i / a.stages) - 1) & 1));
        __syncwarp();  // on a timeout the error bit is set; keep going so every wait stays bounded
      }
      uint8_t* buf = stages + st * a.stage_bytes;
      const TileSpans ts = tile_spans(a, S, i);
      if (lane == 0) {
        // weight bytes first: they are the long pole
        uintptr_t lo, hi;
        uint32_t bytes = 0;
        bulk_window(ts.s0, ts.b0, ts.e0, &lo, &hi);
        bytes += hi > lo ? (uint32_t)(hi - lo) : 0u;
        if (ts.s1.g0) {
          bulk_window(ts.s1, ts.b1, ts.e1, &lo, &hi);
          bytes += hi > lo ? (uint32_t)(hi - lo) : 0u;
        }
        mbar_arrive_expect_tx(&full[st], bytes);
        issue_span(buf, ts.s0, ts.b0, ts.e0, &full[st]);
        if (ts.s1.g0) issue_span(buf + a.half, ts.s1, ts.b1, ts.e1, &full[st]);
        if (i == 0) stamp(a.trace, kEvProducerFirst);
        if (i == ntiles - 1) stamp(a.trace, kEvProducerLast);
      }
      {
        // the tile's bias values: phase 1 gate [0, 12) and up [12, 24); phase 2 down [0, 24)
        const Tile tl = S.tiles[i];
        const int el = S.slot_expert[tl.slot] - p.expert_lo;
        const int nv = tl.r1 - tl.r0;
        float bv = 0.f;
        if (tl.phase == 1) {
          if (lane < 12 && lane < nv && p.gate_b) bv = __ldg(p.gate_b + (int64_t)el * F + tl.r0 + lane);
          if (lane >= 12 && lane < 24 && lane - 12 < nv && p.up_b)
            bv = __ldg(p.up_b + (int64_t)el * F + tl.r0 + lane - 12);
        } else if (lane < nv && lane < kTileCols && p.down_b) {
          bv = __ldg(p.down_b + (int64_t)el * H + tl.r0 + lane);
        }
        if (lane < kTileCols) stage_bias[st * kTileCols + lane] = bv;
      }
      if (span_has_ragged(ts.s0, ts.b0, ts.e0)) copy_ragged(buf, ts.s0, ts.b0, ts.e0, lane);
      if (ts.s1.g0 && span_has_ragged(ts.s1, ts.b1, ts.e1)) copy_ragged(buf + a.half, ts.s1, ts.b1, ts.e1, lane);
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[st]);  // release: biases and ragged bytes are visible
    }
    return;
  }

  // ================================================================= consumer warps
  const int gi = warp % kGroups, kc = warp / kGroups;
  const int g = lane >> 2, q = lane & 3;
  float* sc = sc_base + warp * a.sc_stride;
  bool phase2_started = false;

  auto phase_boundary = [&]() {
    // every activation row of every CTA is written -> build the phase-2 operands
    named_sync(1, kComputeThreads);
    if (tid == 0) {
      stamp(a.trace, kEvPhase1End);
      S.ok = grid_barrier_thread0(a.bar, (unsigned)G);
      stamp(a.trace, kEvBarrier2);
    }
    named_sync(1, kComputeThreads);
    const int np = S.npairs;
    if (kMma) {
      // per-pair scale from the maxima the phase-1 epilogues recorded
      if (tid < np) {
        const int sg = xsplit_sigma(__uint_as_float(__ldcg(a.amax + tid)));
        S.fac_pair[tid] = ldexpf(1.0f, 1 - sg);
        S.sig_pair[tid] = sg;
      }
      named_sync(1, kComputeThreads);
      uint4* aimg = reinterpret_cast<uint4*>(region);
      const int ps = xfrag_part_stride_u4(a.nb_f);
      const int per_pair = a.nb_f * 4;
      for (int it = tid; it < np * per_pair; it += kComputeThreads) {
        const int pr = it / per_pair, i = it - pr * per_pair;
        const int b = i >> 2, qq = i & 3;
        const float scl = ldexpf(1.0f, S.sig_pair[pr]);
        const float* v = a.act + (int64_t)pr * F + 32 * b + 4 * qq;
        const float4 lo4 = __ldcg(reinterpret_cast<const float4*>(v));
        const float4 hi4 = __ldcg(reinterpret_cast<const float4*>(v + 16));
        const float xa[4] = {lo4.x, lo4.y, lo4.z, lo4.w}, xb[4] = {hi4.x, hi4.y, hi4.z, hi4.w};
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float x0 = xa[j] * scl, x1 = xb[j] * scl;
          const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
          __half2 hh = __halves2half2(h0, h1);
          hi[j] = *reinterpret_cast<uint32_t*>(&hh);
          lo[j] = pack_f16x2(x0 - __half2float(h0), x1 - __half2float(h1));
        }
        uint4* img = aimg + pr * xfrag_vec_u4(a.nb_f);
        img[b * 4 + qq] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        img[ps + b * 4 + qq] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
      }
    } else if (kInt) {
      // every pair's activation row as int8 digit planes, one thread per (pair, group)
      uint8_t* xq = reinterpret_cast<uint8_t*>(region);
      float* xsc = reinterpret_cast<float*>(xq + (size_t)np * a.nb_f * kXQG);
      float* xsm = xsc + np * a.nb_f;
      for (int it = tid; it < np * a.nb_f; it += kComputeThreads) {
        const float4* src = reinterpret_cast<const float4*>(a.act + (int64_t)it * 32);  // row pr, group g
        float v[32];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 f = __ldcg(src + j);
          v[4 * j] = f.x; v[4 * j + 1] = f.y; v[4 * j + 2] = f.z; v[4 * j + 3] = f.w;
        }
        group_planes_i8(v, xq + (size_t)it * kXQG, &xsc[it], &xsm[it]);
      }
      for (int pr = tid; pr < np; pr += kComputeThreads) S.fac_pair[pr] = 1.0f;
    } else {
      const int nf = np * F;
      if (!a.act_global)
        for (int i = tid * 4; i < nf; i += kComputeThreads * 4)
          *reinterpret_cast<float4*>(region + i) = __ldcg(reinterpret_cast<const float4*>(a.act + i));
      for (int pr = tid; pr < np; pr += kComputeThreads) S.fac_pair[pr] = 1.0f;
    }
    named_sync(1, kComputeThreads);
    if (tid == 0) stamp(a.trace, kEvPhase2Images);
  };

  for (int i = 0; i < ntiles; ++i) {
    if (i == n1_tiles) {
      phase_boundary();
      phase2_started = true;
    }
    const int st = i % a.stages;
    const uint8_t* buf = stages + st * a.stage_bytes;
    const Tile tl = S.tiles[i];
    const TileSpans ts = tile_spans(a, S, i);
    mbar_wait_bounded(&full[st], (uint32_t)((i / a.stages) & 1));
    if (i == 0 && tid == 0) stamp(a.trace, kEvFirstTile);
    const int j = tl.slot;
    const int el = S.slot_expert[j] - p.expert_lo;
    const int pr0 = S.slot_pair0[j], nt = S.slot_pair0[j + 1] - pr0;
    const int nvalid = tl.r1 - tl.r0;
    const uint8_t* s0base = buf + (reinterpret_cast<uintptr_t>(ts.s0.g0) & 15);
    const uint8_t* s1base = buf + a.half + (reinterpret_cast<uintptr_t>(ts.s1.g0) & 15);
    const int rb = tl.phase == 1 ? a.rb_h : a.rb_f;
    const int nb = tl.phase == 1 ? a.nb_h : a.nb_f;
    float* red = red_base + (i & 1) * kRedFloats;
    const int nlive = tl.phase == 1 ? (nvalid + 3) / 4 : (nvalid + 7) / 8;  // live row-groups
    const bool group_live = gi < nlive;

    if (group_live) {
      if (kMma) {
        const int b0 = (nb * kc) / kKChunks, b1 = (nb * (kc + 1)) / kKChunks;
        // this warp's scales: 8 rows x (b1 - b0) blocks, block-major
        for (int it = lane; it < 8 * (b1 - b0); it += 32) {
          const int r = it & 7, b = b0 + (it >> 3);
          const uint8_t* rp = tile_row(tl.phase, 8 * gi + r, s0base, s1base, nvalid, rb);
          sc[(b - b0) * 8 + r] = e8m0_half_scale(rp[17 * b]);
        }
        __syncwarp();
        const uint8_t* rowg = tile_row(tl.phase, 8 * gi + g, s0base, s1base, nvalid, rb);
        const uint4* img;
        int img_stride;
        if (tl.phase == 1) {
          img = ximg;
          img_stride = xfrag_vec_u4(a.nb_h);
        } else {
          img = reinterpret_cast<const uint4*>(region) + pr0 * xfrag_vec_u4(a.nb_f);
          img_stride = xfrag_vec_u4(a.nb_f);
        }
        const int ps = xfrag_part_stride_u4(nb);
        // x-part xp -> (token slot xp/2, part xp%2)
        auto xrow = [&](int xp) -> const uint4* {
          const int ti = xp >> 1;
          if (ti >= nt) return nullptr;
          const int tokslot = tl.phase == 1 ? S.pair_token[pr0 + ti] : ti;
          return img + tokslot * img_stride + (xp & 1) * ps;
        };
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        mxfp4_group_mma(rowg, xrow(g), NT > 4 ? xrow(g + 8) : nullptr, b0, b1, q, sc - b0 * 8, 8, 0, acc);
        float* rr = red + (kc * kTileCols + 8 * gi + 2 * q) * 16;
        rr[g] = acc[0];
        rr[16 + g] = acc[1];
        rr[g + 8] = acc[2];
        rr[16 + g + 8] = acc[3];
      } else if (kInt) {
        int tok[NT];
        const uint8_t* xq;
        int ng;
        if (tl.phase == 1) {
#pragma unroll
          for (int t = 0; t < NT; ++t) tok[t] = t < nt ? S.pair_token[pr0 + t] : 0;
          xq = reinterpret_cast<const uint8_t*>(ximg);
          ng = a.nb_h;
        } else {
#pragma unroll
          for (int t = 0; t < NT; ++t) tok[t] = pr0 + t;
          xq = reinterpret_cast<const uint8_t*>(region);
          ng = a.nb_f;
        }
        const int nrow = tl.phase == 1 ? T : S.npairs;  // planes' rows: tokens or pairs
        const float* xsc = reinterpret_cast<const float*>(xq + (size_t)nrow * ng * kXQG);
        const bool rows16 = ((reinterpret_cast<uintptr_t>(s0base) | reinterpret_cast<uintptr_t>(s1base) | (uintptr_t)rb) & 15) == 0;
        unit_int8<FMT, NT>(tl.phase, gi, kc, s0base, s1base, nvalid, rb, ng, xq, ng * kXQG, xsc, xsc + nrow * ng,
                           tok, nt, red, lane, rows16);
      } else {
        int tok[NT];
        const float* x;
        int64_t xs;
        if (tl.phase == 1) {
#pragma unroll
          for (int t = 0; t < NT; ++t) tok[t] = t < nt ? S.pair_token[pr0 + t] : 0;
          x = h;
          xs = H;
        } else {
#pragma unroll
          for (int t = 0; t < NT; ++t) tok[t] = t;
          // rows written by every CTA's phase-1 epilogue before the grid barrier; this SM has not
          // read them before, so its loads miss L1 and see L2
          x = (a.act_global ? a.act : region) + (int64_t)pr0 * F;
          xs = F;
        }
        unit_cuda_core<FMT, NT>(tl.phase, gi, kc, s0base, s1base, nvalid, rb, nb, x, xs, tok, nt, red, lane);
      }
    }
    named_sync(2 + gi, 4 * 32);  // the group's four K-chunk partials are in `red`
    const float* tb = stage_bias + st * kTileCols;
    if (group_live) {
      // epilogue of group gi by its 128 threads (fixed item -> thread map)
      const int gt = kc * 32 + lane;
      if (tl.phase == 1) {
        const int nn = min(4, nvalid - 4 * gi);
        for (int it = gt; it < nn * nt; it += 128) {
          const int jn = it / nt, ti = it - jn * nt;
          const int col = 8 * gi + 2 * jn;
          float gs = 0.f, us = 0.f;
#pragma unroll
          for (int kk = 0; kk < kKChunks; ++kk) {
            const float* rg = red + (kk * kTileCols + col) * 16;
            gs += rg[2 * ti] + rg[2 * ti + 1];
            us += rg[16 + 2 * ti] + rg[16 + 2 * ti + 1];
          }
          const int tokid = S.pair_token[pr0 + ti];
          const float fac = S.fac_tok[tokid];
          const int neuron = tl.r0 + 4 * gi + jn;
          float gv = gs * fac, uv = us * fac;
          if (p.gate_b) gv = __fadd_rn(gv, tb[4 * gi + jn]);
          if (p.up_b) uv = __fadd_rn(uv, tb[12 + 4 * gi + jn]);
          const float av = activate(p.act_mode, gv, uv, p.alpha, p.limit);
          a.act[(int64_t)(pr0 + ti) * F + neuron] = av;
          if (kMma) atomicMax(a.amax + pr0 + ti, __float_as_uint(fabsf(av)));
        }
      } else {
        const int nr = min(8, nvalid - 8 * gi);
        for (int it = gt; it < nr * nt; it += 128) {
          const int r = it / nt, ti = it - r * nt;
          const int col = 8 * gi + r;
          float ys = 0.f;
#pragma unroll
          for (int kk = 0; kk < kKChunks; ++kk) {
            const float* rg = red + (kk * kTileCols + col) * 16;
            ys += rg[2 * ti] + rg[2 * ti + 1];
          }
          const int row = tl.r0 + col;
          float y = ys * S.fac_pair[pr0 + ti];
          if (p.down_b) y = __fadd_rn(y, tb[col]);
          float& o = o_acc[S.pair_token[pr0 + ti] * a.rows_cta_max + (row - ra)];
          o = __fadd_rn(o, __fmul_rn(S.pair_w[pr0 + ti], y));
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);  // stage bytes and biases no longer needed by this warp
  }
  if (!phase2_started) phase_boundary();  // no phase-2 tile here; still take part in the barrier

  // ---- output rows of this CTA: out = x + o (or o)
  named_sync(1, kComputeThreads);
  if (tid == 0) stamp(a.trace, kEvTilesEnd);
  const int rb_end = (int)((int64_t)H * (c + 1) / G);
  for (int qq = tid; qq < T * (rb_end - ra); qq += kComputeThreads) {
    const int t = qq / (rb_end - ra), r = ra + (qq - t * (rb_end - ra));
    const float o = o_acc[t * a.rows_cta_max + (r - ra)];
    p.out[(int64_t)t * H + r] = p.add_residual ? __fadd_rn(p.x[(int64_t)t * H + r], o) : o;
  }
  if (tid == 0) stamp(a.trace, kEvEnd);
}

template <int FMT, int NT>
static int launch_moe(const MoeArgs& a, int grid, size_t smem, cudaStream_t stream) {
  auto kern = moe_layer_kernel<FMT, NT>;
  // the kernel's whole budget, not this launch's size (see dense.cu: graphs replay against the attribute)
  NS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)std::max(smem, (size_t)kMoeSmemBudget)));
  int per_sm = 0;
  NS_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kMoeThreads, smem));
  if (per_sm < 1) return fail(NS_ERR_UNSUPPORTED, "ns_moe_decode_layer: kernel does not fit on an SM");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kMoeThreads);
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

template <int FMT>
static int dispatch_moe_t(const MoeArgs& a, int grid, size_t smem, cudaStream_t s) {
  if (a.p.T == 1) return launch_moe<FMT, 1>(a, grid, smem, s);
  if (a.p.T == 2) return launch_moe<FMT, 2>(a, grid, smem, s);
  if (a.p.T <= 4) return launch_moe<FMT, 4>(a, grid, smem, s);
  return launch_moe<FMT, 8>(a, grid, smem, s);
}


// Trace buffer per device (host-side table, set by ns_moe_set_trace).
static unsigned long long* g_trace_buf[64] = {nullptr};
static size_t g_trace_bytes[64] = {0};
static int trace_slot() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  return dev;
}

}  // namespace ns

#include "moe_tc.cu"

namespace ns {

// Kernel choice: 0 = tensor-core kernel where the layer qualifies, 1 = always the
// CUDA-core / mma.sync kernel, 2 = tensor-core kernel or NS_ERR_UNSUPPORTED.
static int g_moe_path = 0;

struct MoePlan {
  size_t ws_logits, ws_act, ws_total;
  int pairs_max;
  bool tc_ok;
  TcPlan tp;
};

static int moe_validate(const ns_moe_layer_t* p, MoePlan* plan) {
  if (!p) return fail(NS_ERR_INVALID, "ns_moe: null parameters");
  if (p->T < 1 || p->T > NS_MAX_TOKENS) return fail(NS_ERR_INVALID, "ns_moe: T=%d outside 1..%d", p->T, NS_MAX_TOKENS);
  if (p->n_expert < 1 || p->n_expert > NS_MAX_EXPERTS)
    return fail(NS_ERR_INVALID, "ns_moe: n_expert=%d outside 1..%d", p->n_expert, NS_MAX_EXPERTS);
  if (p->k < 1 || p->k > NS_MAX_TOPK || p->k > p->n_expert)
    return fail(NS_ERR_INVALID, "ns_moe: k=%d outside 1..min(%d, n_expert)", p->k, NS_MAX_TOPK);
  if (p->expert_lo < 0 || p->expert_hi > p->n_expert || p->expert_lo >= p->expert_hi)
    return fail(NS_ERR_INVALID, "ns_moe: bad local expert range [%d, %d)", p->expert_lo, p->expert_hi);
  if (p->H <= 0 || p->F <= 0 || p->H % 32 || p->F % 32)
    return fail(NS_ERR_INVALID, "ns_moe: H=%d and F=%d must be positive multiples of 32", p->H, p->F);
  if (p->route_mode != NS_ROUTE_TOPK_SOFTMAX && p->route_mode != NS_ROUTE_SOFTMAX_TOPK_NORM)
    return fail(NS_ERR_INVALID, "ns_moe: bad route mode %d", p->route_mode);
  if (p->act_mode != NS_ACT_CLAMPED_SWIGLU && p->act_mode != NS_ACT_SILU_MUL)
    return fail(NS_ERR_INVALID, "ns_moe: bad activation mode %d", p->act_mode);
  if (!float_type_ok(p->router_dtype)) return fail(NS_ERR_INVALID, "ns_moe: bad router dtype %d", p->router_dtype);
  if (p->ggml_type != NS_GGML_MXFP4 && p->ggml_type != NS_GGML_Q8_0 && p->ggml_type != NS_GGML_Q4_K &&
      p->ggml_type != NS_GGML_Q6_K)
    return fail(NS_ERR_UNSUPPORTED, "ns_moe: expert type %d has no fused kernel", p->ggml_type);
  for (int i = 0; i < NS_L2_PREFETCH_RANGES; ++i)
    if (p->l2.bytes[i] && (reinterpret_cast<uintptr_t>(p->l2.ptr[i]) & 15))
      return fail(NS_ERR_INVALID, "ns_moe: L2 prefetch range %d not 16-byte aligned", i);
  if (row_bytes_of(p->ggml_type, p->H) < 0 || row_bytes_of(p->ggml_type, p->F) < 0)
    return fail(NS_ERR_INVALID, "ns_moe: H=%d / F=%d not whole blocks of type %d", p->H, p->F, p->ggml_type);
  plan->pairs_max = p->T * p->k;
  plan->ws_logits = align_up((size_t)p->T * p->n_expert * 4, 256);
  plan->ws_act = align_up((size_t)plan->pairs_max * p->F * 4, 256);
  plan->ws_total = kWsHeader + plan->ws_logits + plan->ws_act;
  plan->tc_ok = moe_tc_eligible(p);
  if (plan->tc_ok) {
    moe_tc_plan(p, kTcGridMax, &plan->tp);
    plan->ws_total = std::max(plan->ws_total, plan->tp.ws_total);
  }
  return NS_OK;
}

// Shared-memory layout of one launch; returns total bytes, or 0 if it cannot fit.
static size_t moe_layout(const ns_moe_layer_t* p, const MoePlan& plan, int grid, MoeArgs* a,
                         bool act_global = false) {
  const bool mma = p->ggml_type == NS_GGML_MXFP4;
  const bool i8 = moe_int8_path(p->ggml_type, p->T);
  a->act_global = act_global && !mma && !i8;
  const int nb_h = p->H / 32, nb_f = p->F / 32;
  // region: phase 1 = h (+ h images or int8 planes), phase 2 = activation images, int8 planes (or
  // fp32 activations)
  const size_t img_h = (size_t)2 * (nb_h * 4 + 4) * 16, img_f = (size_t)2 * (nb_f * 4 + 4) * 16;
  const size_t h_bytes = align_up((size_t)p->T * p->H * 4, 128);
  const size_t pl_h = (size_t)p->T * nb_h * (kXQG + 8), pl_f = (size_t)plan.pairs_max * nb_f * (kXQG + 8);
  const size_t r1 = h_bytes + (mma ? p->T * img_h : i8 ? pl_h : 0);
  const size_t r2 = mma ? plan.pairs_max * img_f : i8 ? pl_f : a->act_global ? 0 : (size_t)plan.pairs_max * p->F * 4;
  const size_t region = align_up(std::max(r1, r2), 128);
  a->rows_cta_max = (p->H + grid - 1) / grid + 1;
  const size_t oacc = align_up((size_t)p->T * a->rows_cta_max * 4, 128);
  const size_t red = (size_t)2 * kRedFloats * 4;
  const int max_chunk_blocks = (std::max(nb_h, nb_f) + kKChunks - 1) / kKChunks + 1;
  a->sc_stride = mma ? 8 * max_chunk_blocks : 0;
  const size_t scb = align_up((size_t)kComputeWarps * a->sc_stride * 4, 128);
  const size_t fixed = region + oacc + red + scb + 2 * kMaxStages * 8 + kMaxStages * kTileCols * 4 +
                       sizeof(MoeShared) + 256;
  const int rb_h = (int)row_bytes_of(p->ggml_type, p->H), rb_f = (int)row_bytes_of(p->ggml_type, p->F);
  if (fixed >= (size_t)kMoeSmemBudget) return 0;
  const size_t avail = kMoeSmemBudget - fixed;
  // tiles: phase 1 up to 12 neurons (two spans), phase 2 up to 24 rows
  int stages = kMaxStages;
  int tn = 12, tr = 24;
  auto stage_of = [&](int n1, int n2) {
    size_t hf = align_up((size_t)n1 * rb_h + 48, 16);
    return align_up(std::max(2 * hf, (size_t)n2 * rb_f + 48), 128);
  };
  while (a->act_global && stages >= 2 && stage_of(tn, tr) * stages > avail) {
    // many activation rows (T x k large): keep tiles wide, since the per-CTA tile list grows as
    // they narrow; shrink the side that sets the stage size, and drop to 2 stages first
    const bool p1_dominates = 2 * align_up((size_t)tn * rb_h + 48, 16) >= (size_t)tr * rb_f + 48;
    if (stages > 3) --stages;
    else if (p1_dominates && tn > 8) tn -= 4;
    else if (!p1_dominates && tr > 16) tr -= 8;
    else if (stages > 2) --stages;
    else if (p1_dominates && tn > 1) tn = tn > 4 ? tn - 4 : tn - 1;
    else if (!p1_dominates && tr > 1) tr = tr > 8 ? tr - 8 : tr - 1;
    else --stages;
  }
  // dp4a consumers: whole tiles (every consumer warp busy) on two stages rather than narrower tiles
  // on three (Qwen3-235B shape: 16-row tiles on three stages left a third of the consumer warps idle;
  // phase 1 took 36 us against 25 us with 24-row tiles on two)
  if (i8 && stage_of(tn, tr) * 3 > avail && stage_of(tn, tr) * 2 <= avail) stages = 2;
  while (stages >= 2 && stage_of(tn, tr) * stages > avail) {
    if (stages > 3) {
      --stages;
    } else if (tn > 4 || tr > 8) {
      if (tn > 4) tn -= 4;
      if (tr > 8) tr -= 8;
    } else if (tn > 1 || tr > 1) {
      tn = std::max(1, tn - 1);
      tr = std::max(1, tr - 1);
    } else {
      --stages;
    }
  }
  if (stages < 2) return 0;
  a->stages = stages;
  a->tn = tn;
  a->tr = tr;
  a->half = (int)align_up((size_t)tn * rb_h + 48, 16);
  a->stage_bytes = (int)stage_of(tn, tr);
  a->nb_h = nb_h;
  a->nb_f = nb_f;
  a->off_oacc = (int)region;
  a->off_red = (int)(region + oacc);
  a->off_sc = (int)(region + oacc + red);
  a->off_stages = (int)align_up(region + oacc + red + scb, 128);
  a->off_bars = a->off_stages + stages * a->stage_bytes;
  a->off_bias = a->off_bars + 2 * kMaxStages * 8;
  a->off_shared = (int)align_up((size_t)a->off_bias + kMaxStages * kTileCols * 4, 16);
  return (size_t)a->off_shared + sizeof(MoeShared);
}

}  // namespace ns

extern "C" int ns_moe_route(const void* h, int h_dtype, int T, int H, const void* w, int w_dtype, const float* b,
                            int E, int k, int mode, int32_t* ids, float* weights, float* logits, ns_stream_t stream) {
  using namespace ns;
  if (T < 1 || H < 1 || E < 1 || E > NS_MAX_EXPERTS || k < 1 || k > NS_MAX_TOPK || k > E)
    return fail(NS_ERR_INVALID, "ns_moe_route: bad shape T=%d H=%d E=%d k=%d", T, H, E, k);
  if (!float_type_ok(h_dtype) || !float_type_ok(w_dtype))
    return fail(NS_ERR_INVALID, "ns_moe_route: bad dtypes h=%d w=%d", h_dtype, w_dtype);
  if (mode != NS_ROUTE_TOPK_SOFTMAX && mode != NS_ROUTE_SOFTMAX_TOPK_NORM)
    return fail(NS_ERR_INVALID, "ns_moe_route: bad mode %d", mode);
  if (!h || !w || !ids || !weights || !logits)
    return fail(NS_ERR_INVALID, "ns_moe_route: null pointer (logits buffer is required as scratch)");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int warps = T * E;
  route_logits_kernel<<<(warps + 7) / 8, 256, 0, s>>>(h, h_dtype, T, H, w, w_dtype, b, E, logits);
  NS_CUDA_TRY(cudaGetLastError());
  const int wpb = 4;
  const size_t smem = (size_t)wpb * (NS_MAX_EXPERTS + 2 * NS_MAX_TOPK) * 4;
  route_select_kernel<<<(T + wpb - 1) / wpb, wpb * 32, smem, s>>>(logits, T, E, k, mode, ids, weights);
  NS_CUDA_TRY(cudaGetLastError());
  return NS_OK;
}

extern "C" int ns_moe_select_kernel(int path) {
  if (path < 0 || path > 2) return ns::fail(NS_ERR_INVALID, "ns_moe_select_kernel: path %d outside 0..2", path);
  ns::g_moe_path = path;
  return NS_OK;
}

extern "C" int ns_moe_set_trace(uint64_t* buf, size_t bytes) {
  using namespace ns;
  int nsm = 0;
  if (buf) {
    int st = num_sms(&nsm);
    if (st) return st;
    if (bytes < (size_t)nsm * NS_TRACE_EVENTS * 8)
      return fail(NS_ERR_SIZE, "ns_moe_set_trace: %zu bytes, need %d", bytes, nsm * NS_TRACE_EVENTS * 8);
  }
  g_trace_buf[trace_slot()] = reinterpret_cast<unsigned long long*>(buf);
  g_trace_bytes[trace_slot()] = buf ? bytes : 0;
  return NS_OK;
}

extern "C" int ns_moe_workspace_bytes(const ns_moe_layer_t* p, size_t* bytes) {
  using namespace ns;
  if (!bytes) return fail(NS_ERR_INVALID, "ns_moe_workspace_bytes: null output");
  MoePlan plan;
  int st = moe_validate(p, &plan);
  if (st) return st;
  size_t need = plan.ws_total;
  // a layer sized for T tokens serves calls with fewer; those may take the tensor-core kernel,
  // whose scratch differs from the CUDA-core kernel's
  for (int t = 1; t < p->T; ++t) {
    ns_moe_layer_t q = *p;
    q.T = t;
    MoePlan pt;
    if (moe_validate(&q, &pt) == NS_OK) need = std::max(need, pt.ws_total);
  }
  *bytes = need;
  return NS_OK;
}

extern "C" int ns_moe_workspace_init(void* workspace, size_t bytes, ns_stream_t stream) {
  if (!workspace) return ns::fail(NS_ERR_INVALID, "ns_moe_workspace_init: null workspace");
  NS_CUDA_TRY(cudaMemsetAsync(workspace, 0, bytes, reinterpret_cast<cudaStream_t>(stream)));
  return NS_OK;
}

namespace ns {

// Builds the launch arguments over a validated, 256-byte aligned scratch of at
// least plan.ws_total bytes and launches the fused layer on `s`.
static int moe_launch(const ns_moe_layer_t* p, const MoePlan& plan, uint8_t* ws, cudaStream_t s) {
  int nsm = 0;
  int st = num_sms(&nsm);
  if (st) return st;
  if (g_moe_path != 1) {
    if (plan.tc_ok && moe_tc_aligned(p) && nsm <= kTcGridMax) {
      TcPlan tp = plan.tp;
      tp.grid = nsm;
      return moe_tc_launch(p, tp, ws, s);
    }
    if (g_moe_path == 2)
      return fail(NS_ERR_UNSUPPORTED, "ns_moe_decode_layer: layer does not qualify for the tensor-core kernel");
  }

  MoeArgs a;
  memset(&a, 0, sizeof a);
  a.p = *p;
  a.rb_h = (int)row_bytes_of(p->ggml_type, p->H);
  a.rb_f = (int)row_bytes_of(p->ggml_type, p->F);
  a.n_local = p->expert_hi - p->expert_lo;
  a.gate_end = p->gate_w + (size_t)a.n_local * p->F * a.rb_h;
  a.up_end = p->up_w + (size_t)a.n_local * p->F * a.rb_h;
  a.down_end = p->down_w + (size_t)a.n_local * p->H * a.rb_f;
  a.bar = reinterpret_cast<unsigned long long*>(ws);
  a.amax = reinterpret_cast<unsigned*>(ws + 64);
  a.logits = reinterpret_cast<float*>(ws + kWsHeader);
  a.act = reinterpret_cast<float*>(ws + kWsHeader + plan.ws_logits);
  a.trace = g_trace_buf[trace_slot()];

  const int grid = nsm;
  size_t smem = moe_layout(p, plan, grid, &a);
  if ((smem == 0 || smem > (size_t)kMoeSmemBudget) && p->ggml_type != NS_GGML_MXFP4)
    smem = moe_layout(p, plan, grid, &a, true);  // activation rows stay in the workspace
  if (smem == 0 || smem > (size_t)kMoeSmemBudget)
    return fail(NS_ERR_UNSUPPORTED,
                "ns_moe_decode_layer: T=%d x k=%d activation rows of F=%d do not fit in shared memory; "
                "use the per-expert GEMV path", p->T, p->k, p->F);
  {
    const int64_t n1 = (int64_t)plan.pairs_max * p->F;
    const int64_t t1 = (n1 / grid + 2) / a.tn + plan.pairs_max + 2;
    const int64_t t2 = ((int64_t)a.rows_cta_max / a.tr + 1) * plan.pairs_max;
    if (t1 + t2 > kMaxTiles) return fail(NS_ERR_UNSUPPORTED, "ns_moe_decode_layer: tile list too long");
  }
  switch (p->ggml_type) {
    case NS_GGML_MXFP4: return dispatch_moe_t<NS_GGML_MXFP4>(a, grid, smem, s);
    case NS_GGML_Q8_0: return dispatch_moe_t<NS_GGML_Q8_0>(a, grid, smem, s);
    case NS_GGML_Q4_K: return dispatch_moe_t<NS_GGML_Q4_K>(a, grid, smem, s);
    default: return dispatch_moe_t<NS_GGML_Q6_K>(a, grid, smem, s);
  }
}

}  // namespace ns

extern "C" int ns_moe_decode_layer(const ns_moe_layer_t* p, void* workspace, size_t workspace_bytes,
                                   ns_stream_t stream) {
  using namespace ns;
  MoePlan plan;
  int st = moe_validate(p, &plan);
  if (st) return st;
  if (!workspace || workspace_bytes < plan.ws_total)
    return fail(NS_ERR_SIZE, "ns_moe_decode_layer: workspace of %zu bytes, need %zu", workspace_bytes, plan.ws_total);
  if (reinterpret_cast<uintptr_t>(workspace) & 255)
    return fail(NS_ERR_INVALID, "ns_moe_decode_layer: workspace must be 256-byte aligned");
  if (!p->x || !p->out || !p->router_w || !p->gate_w || !p->up_w || !p->down_w)
    return fail(NS_ERR_INVALID, "ns_moe_decode_layer: null tensor pointer");
  return moe_launch(p, plan, reinterpret_cast<uint8_t*>(workspace), reinterpret_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------------------------------------
// Allocation-free variant: ns_moe_decode_layer_static.
//
// For callers that cannot allocate device memory per layer call: a plain C / FFI host that binds only this
// library and has no caching allocator of its own, or a decoder whose weight cache has already budgeted
// every free byte of HBM.  cudaMalloc / cudaFree would synchronise the device in the middle of a decode
// step and fragment that budget, so this entry point takes its scratch (grid-barrier counter, activation
// maxima, router logits, expert activations) from one fixed device array linked into the library instead
// of a caller workspace.  It allocates nothing: no cudaMalloc, no cudaFree, no allocating library routine.
//
// Limit: a layer whose scratch (ns_moe_workspace_bytes) exceeds NS_MOE_STATIC_SCRATCH_BYTES is rejected
// with NS_ERR_SIZE before anything is launched.
//
// Set-up: the first call on each device (with that device current) looks the array's address up with
// cudaGetSymbolAddress and clears its header with a synchronous cudaMemset: the grid barrier counter must
// start at zero, so that every launch's barrier targets are whole multiples of the grid.  That first call
// synchronises the device and must come before any stream capture on the device.
//
// One array serves every call on a device: calls that overlap on the GPU (on different streams without an
// ordering between them) race on the scratch and give wrong results.  Calls ordered on one stream are safe.
// ---------------------------------------------------------------------------------------------------------

static __device__ __align__(256) uint8_t g_moe_static_scratch[NS_MOE_STATIC_SCRATCH_BYTES];

namespace ns {

static std::mutex g_static_mu;
static uint8_t* g_static_ptr[64] = {nullptr};

// Address of this device's static scratch; the first call per device resolves and clears it.
static int static_scratch(uint8_t** out) {
  int dev = 0;
  NS_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(NS_ERR_INVALID, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (!g_static_ptr[dev]) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_moe_static_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static MoE scratch)");
    if (reinterpret_cast<uintptr_t>(ptr) & 255)
      return fail(NS_ERR_CUDA, "static MoE scratch at %p is not 256-byte aligned", ptr);
    e = cudaMemset(ptr, 0, kWsHeader);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(static MoE scratch header)");
    e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize after clearing the static MoE scratch");
    g_static_ptr[dev] = static_cast<uint8_t*>(ptr);
  }
  *out = g_static_ptr[dev];
  return NS_OK;
}

}  // namespace ns

extern "C" int ns_moe_decode_layer_static(const ns_moe_layer_t* p, ns_stream_t stream) {
  using namespace ns;
  MoePlan plan;
  int st = moe_validate(p, &plan);
  if (st) return st;
  if (plan.ws_total > (size_t)NS_MOE_STATIC_SCRATCH_BYTES)
    return fail(NS_ERR_SIZE,
                "ns_moe_decode_layer_static: this layer needs %zu bytes of scratch (T=%d, k=%d, F=%d, "
                "n_expert=%d); the static scratch holds %d (NS_MOE_STATIC_SCRATCH_BYTES). "
                "Use ns_moe_decode_layer with a caller workspace",
                plan.ws_total, p->T, p->k, p->F, p->n_expert, NS_MOE_STATIC_SCRATCH_BYTES);
  if (!p->x || !p->out || !p->router_w || !p->gate_w || !p->up_w || !p->down_w)
    return fail(NS_ERR_INVALID, "ns_moe_decode_layer_static: null tensor pointer");
  uint8_t* ws = nullptr;
  st = static_scratch(&ws);
  if (st) return st;
  return moe_launch(p, plan, ws, reinterpret_cast<cudaStream_t>(stream));
}
