// MoE decode step on device: router (ns_moe_route) and the fused layer
// (ns_moe_decode_layer).
//
// The fused layer is ONE cooperative launch of one CTA per SM:
//   1. every CTA: h = RMSNorm(x) into shared memory (redundant, H floats);
//   2. router logits, one expert per CTA (CTA c: experts c, c+G, ...) -> workspace;
//   3. grid barrier; every CTA re-derives top-k + weights from the logits and
//      builds the routed-expert slots (ascending expert id, as the reference
//      walks torch.unique(ids));
//   4. phase 1: the (slot, neuron) space is split evenly over CTAs; a tile is
//      up to TN neurons of one slot: its gate and up rows stream in by bulk
//      copy, the CTA computes gate.h + b, up.h + b and the activation, and
//      writes the activation rows to the workspace;
//   5. grid barrier; phase 2: output rows are split evenly over CTAs; for each
//      row sub-tile the CTA walks the slots in ascending expert order, streams
//      that expert's down rows, and accumulates w * (down.a + b) in the
//      reference's order, then adds the residual.
// Weight copies run ahead across the phase-2 barrier (the ring is filled with
// phase-2 tiles before the barrier wait), and every device wait is bounded.
#include "qdot.cuh"

namespace ns {

constexpr int kMoeThreads = 256;
constexpr int kMoeWarps = kMoeThreads / 32;
constexpr int kMoeStages = 3;
constexpr int kMaxPairs = NS_MAX_TOKENS * NS_MAX_TOPK;  // (slot, token) pairs
constexpr int kMaxTiles = 512;
constexpr int kMoeSmemBudget = 224 * 1024;

// ----------------------------------------------------------------------------- routing helpers

// Top-k of v[0..E) by (value desc, index asc), one warp.  Writes ids/vals to smem arrays.
__device__ void warp_topk(const float* v, int E, int k, int* ids, float* vals, int lane) {
  uint32_t taken[NS_MAX_EXPERTS / 32];
  for (int i = 0; i < NS_MAX_EXPERTS / 32; ++i) taken[i] = 0u;
  for (int j = 0; j < k; ++j) {
    float best = -INFINITY;
    int bi = 0x7FFFFFFF;
    for (int e = lane; e < E; e += 32) {
      if ((taken[e >> 5] >> (e & 31)) & 1u) continue;
      float x = v[e];
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
    taken[bi >> 5] |= 1u << (bi & 31);
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

struct MoeArgs {
  ns_moe_layer_t p;
  int rb_h, rb_f;     // bytes of a gate/up row (K=H) and of a down row (K=F)
  int n_local;
  const uint8_t* gate_end;
  const uint8_t* up_end;
  const uint8_t* down_end;
  float* logits;      // workspace: T x E
  float* act;         // workspace: pairs x F
  unsigned long long* bar;
  int stage_bytes;
  int tn;             // phase-1 neurons per tile
  int tr;             // phase-2 rows per tile
  int region_floats;  // shared region holding h, later the activations
  int rows_cta_max;   // phase-2 output rows per CTA, upper bound
};

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
  int ok;
  float red[kMoeWarps][NS_MAX_TOKENS];
  Tile tiles[kMaxTiles];
  float scratch[NS_MAX_EXPERTS];
};

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Grid-wide barrier on a monotonically increasing 64-bit counter: barrier
// instance n completes when the counter reaches (n+1)*G.  Bounded wait.
__device__ bool grid_barrier(unsigned long long* bar, unsigned G, int* s_ok) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    unsigned long long old = atomicAdd(bar, 1ull);
    unsigned long long target = (old / G + 1ull) * G;
    int ok = 1;
    uint64_t t0 = globaltimer_ns();
    while (ld_acquire_u64(bar) < target) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        raise_device_error(NS_DEVERR_GRID_WAIT);
        ok = 0;
        break;
      }
      __nanosleep(32);
    }
    *s_ok = ok;
  }
  __syncthreads();
  return *s_ok != 0;
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

template <int FMT, int NT>
__global__ void __launch_bounds__(kMoeThreads, 1) moe_layer_kernel(MoeArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const ns_moe_layer_t& p = a.p;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, c = blockIdx.x;
  const int T = p.T, H = p.H, F = p.F, E = p.n_expert, k = p.k;

  float* region = reinterpret_cast<float*>(smem);                       // h, then activations
  float* o_acc = region + a.region_floats;                              // T x rows_cta_max
  uint8_t* stages = reinterpret_cast<uint8_t*>(o_acc + ((T * a.rows_cta_max + 31) / 32) * 32);
  uint64_t* bars = reinterpret_cast<uint64_t*>(stages + kMoeStages * a.stage_bytes);
  MoeShared& S = *reinterpret_cast<MoeShared*>(bars + kMoeStages);

  if (tid == 0) {
    for (int s = 0; s < kMoeStages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }

  // ---- 1. h = RMSNorm(x) (or x) into shared memory
  for (int t = 0; t < T; ++t) {
    float ss = 0.f;
    for (int i = tid; i < H; i += kMoeThreads) {
      float v = p.x[(int64_t)t * H + i];
      region[t * H + i] = v;
      ss = fmaf(v, v, ss);
    }
    ss = warp_sum(ss);
    if (lane == 0) S.red[warp][t] = ss;
  }
  __syncthreads();
  if (p.norm_w) {
    for (int t = 0; t < T; ++t) {
      float ss = 0.f;
      for (int w = 0; w < kMoeWarps; ++w) ss += S.red[w][t];
      const float r = 1.0f / sqrtf(ss / (float)H + p.rms_eps);
      for (int i = tid; i < H; i += kMoeThreads)
        region[t * H + i] = __fmul_rn(__fmul_rn(region[t * H + i], r), p.norm_w[i]);
    }
  }
  __syncthreads();

  // ---- 2. router logits: CTA c computes experts c, c+G, ...
  for (int e = c; e < E; e += G) {
    float s[NS_MAX_TOKENS];
#pragma unroll
    for (int t = 0; t < NS_MAX_TOKENS; ++t) s[t] = 0.f;
    for (int i = tid; i < H; i += kMoeThreads) {
      const float wv = load_float(p.router_w, p.router_dtype, (int64_t)e * H + i);
#pragma unroll
      for (int t = 0; t < NS_MAX_TOKENS; ++t)
        if (t < T) s[t] = fmaf(region[t * H + i], wv, s[t]);
    }
#pragma unroll
    for (int t = 0; t < NS_MAX_TOKENS; ++t) {
      if (t < T) {
        float v = warp_sum(s[t]);
        if (lane == 0) S.red[warp][t] = v;
      }
    }
    __syncthreads();
    if (tid < T) {
      float v = 0.f;
      for (int w = 0; w < kMoeWarps; ++w) v += S.red[w][tid];
      if (p.router_b) v += p.router_b[e];
      a.logits[(int64_t)tid * E + e] = v;
    }
    __syncthreads();
  }

  // ---- 3. barrier, then routing + slots (identical in every CTA)
  grid_barrier(a.bar, (unsigned)G, &S.ok);
  for (int t = 0; t < T; ++t) {
    if (warp == 0) {
      for (int e = lane; e < E; e += 32) S.scratch[e] = __ldcg(a.logits + (int64_t)t * E + e);
      __syncwarp();
      // Qwen mode overwrites scratch with probabilities; it holds a private copy
      warp_route(S.scratch, E, k, p.route_mode, S.ids[t], S.w[t], S.scratch, lane);
    }
    __syncthreads();
  }
  if (tid == 0) {
    // distinct local experts in ascending order
    int n = 0;
    for (int t = 0; t < T; ++t)
      for (int j = 0; j < k; ++j) {
        int e = S.ids[t][j];
        if (e < p.expert_lo || e >= p.expert_hi) continue;
        int pos = 0;
        while (pos < n && S.slot_expert[pos] < e) ++pos;
        if (pos < n && S.slot_expert[pos] == e) continue;
        for (int q = n; q > pos; --q) S.slot_expert[q] = S.slot_expert[q - 1];
        S.slot_expert[pos] = e;
        ++n;
      }
    int np = 0;
    for (int j = 0; j < n; ++j) {
      S.slot_pair0[j] = np;
      for (int t = 0; t < T; ++t)
        for (int q = 0; q < k; ++q)
          if (S.ids[t][q] == S.slot_expert[j]) {
            S.pair_token[np] = t;
            S.pair_w[np] = S.w[t][q];
            ++np;
          }
    }
    S.slot_pair0[n] = np;
    S.nslots = n;
    S.npairs = np;
    // tiles: phase 1 over the flattened (slot, neuron) space, then phase 2
    int nt = 0;
    const int64_t N1 = (int64_t)n * F;
    int64_t pos = N1 * c / G, end1 = N1 * (c + 1) / G;
    while (pos < end1 && nt < kMaxTiles) {
      int j = (int)(pos / F), n0 = (int)(pos - (int64_t)j * F);
      int64_t lim = (int64_t)n0 + (end1 - pos);
      if (lim > (int64_t)n0 + a.tn) lim = (int64_t)n0 + a.tn;
      if (lim > (int64_t)F) lim = F;
      int n1 = (int)lim;
      S.tiles[nt++] = Tile{1, (short)j, n0, n1};
      pos += n1 - n0;
    }
    S.n1_tiles = nt;
    const int ra = (int)((int64_t)H * c / G), rb = (int)((int64_t)H * (c + 1) / G);
    for (int r0 = ra; r0 < rb; r0 += a.tr)
      for (int j = 0; j < n && nt < kMaxTiles; ++j) S.tiles[nt++] = Tile{2, (short)j, r0, min(rb, r0 + a.tr)};
    S.ntiles = nt;
    if (c == 0) {
      for (int t = 0; t < T; ++t)
        for (int j = 0; j < k; ++j) {
          if (p.ids) p.ids[t * k + j] = S.ids[t][j];
          if (p.weights) p.weights[t * k + j] = S.w[t][j];
        }
    }
  }
  __syncthreads();
  const int nslots = S.nslots, ntiles = S.ntiles;

  // ---- weight streaming: tile i -> stage i % kMoeStages
  const int half = (a.stage_bytes / 2) & ~15;
  auto spans = [&](int i, Span* s0, Span* s1, const uint8_t** e0, const uint8_t** e1, const uint8_t** b0) {
    const Tile tl = S.tiles[i];
    const int el = S.slot_expert[tl.slot] - p.expert_lo;
    if (tl.phase == 1) {
      const int64_t row0 = (int64_t)el * F + tl.r0, row1 = (int64_t)el * F + tl.r1;
      *s0 = Span{p.gate_w + row0 * a.rb_h, p.gate_w + row1 * a.rb_h};
      *s1 = Span{p.up_w + row0 * a.rb_h, p.up_w + row1 * a.rb_h};
      *b0 = p.gate_w;
      *e0 = a.gate_end;
      *e1 = a.up_end;
    } else {
      const int64_t row0 = (int64_t)el * H + tl.r0, row1 = (int64_t)el * H + tl.r1;
      *s0 = Span{p.down_w + row0 * a.rb_f, p.down_w + row1 * a.rb_f};
      *s1 = Span{nullptr, nullptr};
      *b0 = p.down_w;
      *e0 = a.down_end;
      *e1 = nullptr;
    }
  };
  auto issue = [&](int i) {
    const int st = i % kMoeStages;
    uint8_t* buf = stages + st * a.stage_bytes;
    Span s0, s1;
    const uint8_t *e0, *e1, *b0;
    spans(i, &s0, &s1, &e0, &e1, &b0);
    uintptr_t lo, hi;
    uint32_t bytes = 0;
    bulk_window(s0, b0, e0, &lo, &hi);
    bytes += hi > lo ? (uint32_t)(hi - lo) : 0u;
    if (s1.g0) {
      bulk_window(s1, p.up_w, e1, &lo, &hi);
      bytes += hi > lo ? (uint32_t)(hi - lo) : 0u;
    }
    mbar_arrive_expect_tx(&bars[st], bytes);
    issue_span(buf, s0, b0, e0, &bars[st]);
    if (s1.g0) issue_span(buf + half, s1, p.up_w, e1, &bars[st]);
  };
  if (tid == 0)
    for (int i = 0; i < kMoeStages && i < ntiles; ++i) issue(i);

  // phase-2 output accumulators
  for (int i = tid; i < T * a.rows_cta_max; i += kMoeThreads) o_acc[i] = 0.f;

  const int ngroups_h = H / 32, ngroups_f = F / 32;
  constexpr int RN = (NT <= 2) ? 2 : 1;  // phase-1 neurons per warp step (2*RN rows)
  constexpr int R2 = (NT <= 2) ? 4 : 2;  // phase-2 rows per warp step
  const int ra = (int)((int64_t)H * c / G);

  for (int i = 0; i < ntiles; ++i) {
    if (i == S.n1_tiles) {
      // all activations written -> barrier, then stage them in shared memory
      grid_barrier(a.bar, (unsigned)G, &S.ok);
      const int nf = S.npairs * F;
      for (int q = tid * 4; q < nf; q += kMoeThreads * 4)
        *reinterpret_cast<float4*>(region + q) = __ldcg(reinterpret_cast<const float4*>(a.act + q));
      __syncthreads();
    }
    const int st = i % kMoeStages;
    uint8_t* buf = stages + st * a.stage_bytes;
    Span s0, s1;
    const uint8_t *e0, *e1, *b0;
    spans(i, &s0, &s1, &e0, &e1, &b0);
    const bool ok = mbar_wait_bounded(&bars[st], (uint32_t)((i / kMoeStages) & 1));
    const bool rag0 = span_has_ragged(s0, b0, e0);
    const bool rag1 = s1.g0 && span_has_ragged(s1, p.up_w, e1);
    if (rag0 || rag1) {
      if (warp == 0 && rag0) copy_ragged(buf, s0, b0, e0, lane);
      if (warp == 1 && rag1) copy_ragged(buf + half, s1, p.up_w, e1, lane);
      __syncthreads();
    }
    const Tile tl = S.tiles[i];
    const int j = tl.slot;
    const int el = S.slot_expert[j] - p.expert_lo;
    const int pr0 = S.slot_pair0[j], nt = S.slot_pair0[j + 1] - pr0;
    int tok[NT];
    if (ok && tl.phase == 1) {
#pragma unroll
      for (int t = 0; t < NT; ++t) tok[t] = t < nt ? S.pair_token[pr0 + t] : 0;
      const uint8_t* gbase = buf + (reinterpret_cast<uintptr_t>(s0.g0) & 15);
      const uint8_t* ubase = buf + half + (reinterpret_cast<uintptr_t>(s1.g0) & 15);
      const int nn = tl.r1 - tl.r0;
      for (int n = warp * RN; n < nn; n += kMoeWarps * RN) {
        const int nr = min(RN, nn - n);
        const uint8_t* rows[2 * RN];
#pragma unroll
        for (int r = 0; r < RN; ++r) {
          rows[r] = gbase + (int64_t)(n + min(r, nr - 1)) * a.rb_h;
          rows[RN + r] = ubase + (int64_t)(n + min(r, nr - 1)) * a.rb_h;
        }
        float acc[2 * RN][NT];
#pragma unroll
        for (int r = 0; r < 2 * RN; ++r)
#pragma unroll
          for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;
        dot_rows<FMT, NT, 2 * RN>(rows, 2 * RN, ngroups_h, lane, region, H, tok, nt, acc);
#pragma unroll
        for (int r = 0; r < RN; ++r) {
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            const float gv = warp_sum(acc[r][t]);
            const float uv = warp_sum(acc[RN + r][t]);
            if (lane == 0 && r < nr && t < nt) {
              const int neuron = tl.r0 + n + r;
              float g = gv, u = uv;
              if (p.gate_b) g = __fadd_rn(g, p.gate_b[(int64_t)el * F + neuron]);
              if (p.up_b) u = __fadd_rn(u, p.up_b[(int64_t)el * F + neuron]);
              a.act[(int64_t)(pr0 + t) * F + neuron] = activate(p.act_mode, g, u, p.alpha, p.limit);
            }
          }
        }
      }
    } else if (ok) {
#pragma unroll
      for (int t = 0; t < NT; ++t) tok[t] = t;
      const uint8_t* base = buf + (reinterpret_cast<uintptr_t>(s0.g0) & 15);
      const int nn = tl.r1 - tl.r0;
      for (int n = warp * R2; n < nn; n += kMoeWarps * R2) {
        const int nr = min(R2, nn - n);
        const uint8_t* rows[R2];
#pragma unroll
        for (int r = 0; r < R2; ++r) rows[r] = base + (int64_t)(n + min(r, nr - 1)) * a.rb_f;
        float acc[R2][NT];
#pragma unroll
        for (int r = 0; r < R2; ++r)
#pragma unroll
          for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;
        dot_rows<FMT, NT, R2>(rows, nr, ngroups_f, lane, region + (int64_t)pr0 * F, F, tok, nt, acc);
#pragma unroll
        for (int r = 0; r < R2; ++r) {
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            const float v = warp_sum(acc[r][t]);
            if (lane == 0 && r < nr && t < nt) {
              const int row = tl.r0 + n + r;
              float y = v;
              if (p.down_b) y = __fadd_rn(y, p.down_b[(int64_t)el * H + row]);
              float& o = o_acc[S.pair_token[pr0 + t] * a.rows_cta_max + (row - ra)];
              o = __fadd_rn(o, __fmul_rn(S.pair_w[pr0 + t], y));
            }
          }
        }
      }
    }
    __syncthreads();  // stage consumed; o_acc updates visible
    if (tid == 0 && i + kMoeStages < ntiles) issue(i + kMoeStages);
  }
  if (S.n1_tiles == ntiles) {
    // no phase-2 tile ran here; still take part in the second barrier
    grid_barrier(a.bar, (unsigned)G, &S.ok);
  }

  // ---- output rows of this CTA: out = x + o (or o)
  const int rb_end = (int)((int64_t)H * (c + 1) / G);
  for (int q = tid; q < T * (rb_end - ra); q += kMoeThreads) {
    const int t = q / (rb_end - ra), r = ra + (q - t * (rb_end - ra));
    const float o = o_acc[t * a.rows_cta_max + (r - ra)];
    p.out[(int64_t)t * H + r] = p.add_residual ? __fadd_rn(p.x[(int64_t)t * H + r], o) : o;
  }
  (void)nslots;
}

template <int FMT, int NT>
static int launch_moe(const MoeArgs& a, int grid, size_t smem, cudaStream_t stream) {
  auto kern = moe_layer_kernel<FMT, NT>;
  NS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
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

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

struct MoePlan {
  size_t ws_logits, ws_act, ws_total;
  int pairs_max;
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
  if (row_bytes_of(p->ggml_type, p->H) < 0 || row_bytes_of(p->ggml_type, p->F) < 0)
    return fail(NS_ERR_INVALID, "ns_moe: H=%d / F=%d not whole blocks of type %d", p->H, p->F, p->ggml_type);
  plan->pairs_max = p->T * p->k;
  plan->ws_logits = align_up((size_t)p->T * p->n_expert * 4, 256);
  plan->ws_act = align_up((size_t)plan->pairs_max * p->F * 4, 256);
  plan->ws_total = 256 + plan->ws_logits + plan->ws_act;
  return NS_OK;
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

extern "C" int ns_moe_workspace_bytes(const ns_moe_layer_t* p, size_t* bytes) {
  using namespace ns;
  if (!bytes) return fail(NS_ERR_INVALID, "ns_moe_workspace_bytes: null output");
  MoePlan plan;
  int st = moe_validate(p, &plan);
  if (st) return st;
  *bytes = plan.ws_total;
  return NS_OK;
}

extern "C" int ns_moe_workspace_init(void* workspace, size_t bytes, ns_stream_t stream) {
  if (!workspace) return ns::fail(NS_ERR_INVALID, "ns_moe_workspace_init: null workspace");
  NS_CUDA_TRY(cudaMemsetAsync(workspace, 0, bytes, reinterpret_cast<cudaStream_t>(stream)));
  return NS_OK;
}

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
  int nsm = 0;
  st = num_sms(&nsm);
  if (st) return st;

  MoeArgs a;
  a.p = *p;
  a.rb_h = (int)row_bytes_of(p->ggml_type, p->H);
  a.rb_f = (int)row_bytes_of(p->ggml_type, p->F);
  a.n_local = p->expert_hi - p->expert_lo;
  a.gate_end = p->gate_w + (size_t)a.n_local * p->F * a.rb_h;
  a.up_end = p->up_w + (size_t)a.n_local * p->F * a.rb_h;
  a.down_end = p->down_w + (size_t)a.n_local * p->H * a.rb_f;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  a.bar = reinterpret_cast<unsigned long long*>(ws);
  a.logits = reinterpret_cast<float*>(ws + 256);
  a.act = reinterpret_cast<float*>(ws + 256 + plan.ws_logits);

  const int grid = nsm;
  a.rows_cta_max = (p->H + grid - 1) / grid + 1;
  a.region_floats = (int)align_up((size_t)std::max(p->T * p->H, plan.pairs_max * p->F), 32);
  const size_t fixed = (size_t)a.region_floats * 4 + align_up((size_t)p->T * a.rows_cta_max, 32) * 4 +
                       kMoeStages * 8 + sizeof(MoeShared) + 128;
  if (fixed + kMoeStages * 4096 > (size_t)kMoeSmemBudget)
    return fail(NS_ERR_UNSUPPORTED,
                "ns_moe_decode_layer: T=%d x k=%d activation rows of F=%d do not fit in shared memory; "
                "use the per-expert GEMV path", p->T, p->k, p->F);
  a.stage_bytes = (int)std::min<size_t>(48 * 1024, ((kMoeSmemBudget - fixed) / kMoeStages) & ~size_t(15));
  const int half = (a.stage_bytes / 2) & ~15;
  a.tn = (half - 64) / a.rb_h;
  a.tr = (a.stage_bytes - 64) / a.rb_f;
  if (a.tn < 1 || a.tr < 1)
    return fail(NS_ERR_UNSUPPORTED, "ns_moe_decode_layer: rows of %d / %d bytes exceed the %d-byte stage", a.rb_h,
                a.rb_f, a.stage_bytes);
  a.tn = std::min(a.tn, 64);
  a.tr = std::min(a.tr, 64);
  // tile list bound
  {
    const int64_t n1 = (int64_t)plan.pairs_max * p->F;
    const int64_t t1 = (n1 / grid + 2) / a.tn + plan.pairs_max + 2;
    const int64_t t2 = ((int64_t)a.rows_cta_max / a.tr + 1) * plan.pairs_max;
    if (t1 + t2 > kMaxTiles) return fail(NS_ERR_UNSUPPORTED, "ns_moe_decode_layer: tile list too long");
  }
  const size_t smem = (size_t)a.region_floats * 4 + align_up((size_t)p->T * a.rows_cta_max, 32) * 4 +
                      (size_t)kMoeStages * a.stage_bytes + kMoeStages * 8 + sizeof(MoeShared);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (p->ggml_type) {
    case NS_GGML_MXFP4: return dispatch_moe_t<NS_GGML_MXFP4>(a, grid, smem, s);
    case NS_GGML_Q8_0: return dispatch_moe_t<NS_GGML_Q8_0>(a, grid, smem, s);
    case NS_GGML_Q4_K: return dispatch_moe_t<NS_GGML_Q4_K>(a, grid, smem, s);
    default: return dispatch_moe_t<NS_GGML_Q6_K>(a, grid, smem, s);
  }
}
