// ns_attn_block: a GPT-OSS attention block for one decode token as ONE cooperative launch:
//
//   q, k, v = W_{q,k,v} rms_norm(x) + b          (phase A, every CTA a slice of the rows)
//   --- grid barrier ---
//   per (kv head g, key split s): RoPE, KV append, online-softmax partial over the split's keys;
//   the last split of kv head g to finish merges all of them with the sinks (phase B)
//   --- grid barrier ---
//   out = x + W_o attn + b_o                      (phase D, every CTA a slice of the rows)
//
// It is the composition of ns_dense_gemv (q/k/v), ns_attn_decode and ns_dense_gemv (o-proj) --
// the reference's GptOssModel._attention_block (neurostream/model/gpt_oss.py:101-114) -- with the
// kernel boundaries removed.  What the boundaries cost is latency, not bytes: each of the three
// launches streamed its few tens of MB at a quarter of HBM bandwidth, spending its time in ramp-up,
// tail and dependent global round trips.  Here every SM streams ONE ordered byte sequence through
// one ring of shared-memory stages: its q/k/v rows, then the key/value history of its attention
// split, then its o-proj rows.  A producer warp issues the 1-D bulk copies (TMA engine) as stages
// free up, independently of the phases; all of it is static data (weights, cache slots below pos),
// so it starts before griddepcontrol.wait and runs on while the compute warps wait at grid
// barriers -- the o-proj weights are in shared memory by the time phase D starts.
//
// Compute warps (8) do the arithmetic of the standalone kernels: K split over 256 threads with the
// activations in registers and a butterfly row reduction for the projections; per split, lane j
// scores keys j and j+32 of a 64-key block for the warp's query head (rows read at rotated column
// offsets, so that 16-byte loads of 256-byte rows stay free of bank conflicts) and accumulates
// p * V.  Every grid barrier and every stage wait is bounded; a wait that runs out raises a device
// error bit, the CTA stops computing, lets the copies it issued land and returns.
//
// Stream order: the kernel lets its dependents launch only after its own griddepcontrol.wait (the
// chain invariant of this library: when a kernel starts, the kernel two places before it in the
// stream has completed), and reads x only after that wait.

namespace ns {

constexpr int kAbWarps = 8;
constexpr int kAbThreads = (kAbWarps + 1) * 32;
constexpr int kAbTileRows = 8;
constexpr int kAbStages = 3;
constexpr int kAbStageBytes = 64 * 1024;      // 8 rows of K <= 4096 bf16, or one 64-key K+V block
constexpr int kAbKeyBlock = 64;
constexpr int kAbHd = 64;
constexpr int kAbMaxRep = 8;
constexpr int kAbMaxRows = 64;                // rows of one projection one CTA may own (staged epilogue data)
constexpr int kAbPartStride = 2 + kAbHd;      // max, sum, output per (kv head, split, query head)

struct AbArgs {
  ns_attn_block_t p;
  int qd, kvd, qkv_rows;                     // q rows, k (= v) rows, q + k + v rows
  int splits;                                // key splits per kv head
  unsigned long long* bar;                   // grid barrier counter (workspace)
  float* yqkv;                               // q, k, v (workspace)
  float* part;                               // [kv head][split][query head][2 + hd] (workspace)
  float* attn;                               // merged attention output, n_head * hd (workspace)
  unsigned* cnt;                             // per kv head: splits done (reset by the merging CTA)
  unsigned long long* trace;                 // per-CTA phase stamps (ns_moe_set_trace), or null
};

// Phase stamps of the tracer (per CTA, NS_TRACE_EVENTS slots).
enum { kAbEvStart = 0, kAbEvNorm, kAbEvPhaseA, kAbEvBar1, kAbEvPhaseB, kAbEvBar2, kAbEvEnd };

// Tiles of one CTA's byte stream: 0 = q/k/v rows, 1 = a key/value block, 2 = o-proj rows.
struct AbPlan {
  int a0, a1;          // q/k/v rows [a0, a1)
  int d0, d1;          // o-proj rows [d0, d1)
  int item;            // attention work item (kv head * splits + split), or -1
  int g, s, j0, j1;    // its kv head, split and keys [j0, j1)
  int nA, nB, nD;      // tiles of each kind
};

__device__ __forceinline__ AbPlan ab_plan(const AbArgs& a, int pos, int c, int G) {
  AbPlan q;
  q.a0 = (int)((int64_t)a.qkv_rows * c / G);
  q.a1 = (int)((int64_t)a.qkv_rows * (c + 1) / G);
  q.d0 = (int)((int64_t)a.p.H * c / G);
  q.d1 = (int)((int64_t)a.p.H * (c + 1) / G);
  const int items = a.p.n_head_kv * a.splits;
  q.item = c < items ? c : -1;
  q.g = q.item >= 0 ? q.item / a.splits : 0;
  q.s = q.item >= 0 ? q.item % a.splits : 0;
  const int k_lo = a.p.window > 0 ? max(0, pos - a.p.window + 1) : 0;
  const int n_keys = pos - k_lo + 1;
  q.j0 = k_lo + (int)((int64_t)n_keys * q.s / a.splits);
  q.j1 = k_lo + (int)((int64_t)n_keys * (q.s + 1) / a.splits);
  q.nA = (q.a1 - q.a0 + kAbTileRows - 1) / kAbTileRows;
  q.nB = q.item >= 0 ? (q.j1 - q.j0 + kAbKeyBlock - 1) / kAbKeyBlock : 0;
  q.nD = (q.d1 - q.d0 + kAbTileRows - 1) / kAbTileRows;
  return q;
}

// Bulk copy of [src, src + n) into dst in pieces of <= 16 KB (n a multiple of 16), completing on bar.
__device__ __forceinline__ void ab_copy(uint8_t* dst, const uint8_t* src, uint32_t n, uint64_t* bar) {
  while (n > 0) {
    const uint32_t m = min(n, 16384u);
    bulk_g2s(dst, src, m, bar);
    dst += m;
    src += m;
    n -= m;
  }
}

// Grid barrier among the compute warps of all CTAs (counter targets are whole multiples of the
// grid).  Returns false if the wait ran out (device error raised).
__device__ __forceinline__ bool ab_grid_sync(unsigned long long* bar, int G, int tid, volatile int* ok) {
  named_sync(1, kAbWarps * 32);
  if (tid == 0) {
    // one release add (orders this CTA's writes, which the CTA barrier gathered, before it), then
    // acquire loads until every CTA has arrived
    unsigned long long old;
    asm volatile("atom.add.release.gpu.global.u64 %0, [%1], 1;" : "=l"(old) : "l"(bar) : "memory");
    const unsigned long long target = (old / (unsigned)G + 1ull) * (unsigned)G;
    if (ld_acquire_u64(bar) < target) {
      const uint64_t t0 = globaltimer_ns();
      while (ld_acquire_u64(bar) < target) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          raise_device_error(NS_DEVERR_GRID_WAIT);
          *ok = 0;
          break;
        }
      }
    }
  }
  named_sync(1, kAbWarps * 32);
  return *ok != 0;
}

// One projection tile: 8 rows x K (bf16 at st, row pitch K*2 bytes) against this thread's NCH
// 8-element chunks of the activations (xv), summed over the 256 compute threads; returns the row
// total in threads 0..7 (thread r holds row r).  red: [2][8 warps][8 rows] scratch, buffer rb.
template <int NCH>
__device__ __forceinline__ float ab_tile(const uint8_t* st, int K, int rows, const float (&xv)[NCH][8], float* red,
                                         int rbuf, int tid, int lane, int warp) {
  const int nchunk = K / 8;
  float acc[kAbTileRows];
#pragma unroll
  for (int r = 0; r < kAbTileRows; ++r) acc[r] = 0.f;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int ch = tid + c * kAbWarps * 32;
    if (ch < nchunk) {
#pragma unroll
      for (int r = 0; r < kAbTileRows; ++r) {
        if (r >= rows) break;
        const uint4 w = *reinterpret_cast<const uint4*>(st + (size_t)r * K * 2 + (size_t)ch * 16);
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[r] = fmaf(__uint_as_float(ww[j] << 16), xv[c][2 * j], acc[r]);
          acc[r] = fmaf(__uint_as_float(ww[j] & 0xFFFF0000u), xv[c][2 * j + 1], acc[r]);
        }
      }
    }
  }
  const float v = reduce8_rows(acc, lane);
  float* rb = red + rbuf * kAbWarps * kAbTileRows;
  if ((lane & 3) == 0) rb[warp * kAbTileRows + dense_row_of(lane)] = v;
  named_sync(1, kAbWarps * 32);
  float sum = 0.f;
  if (tid < kAbTileRows)
#pragma unroll
    for (int w = 0; w < kAbWarps; ++w) sum += rb[w * kAbTileRows + tid];
  return sum;
}

struct AbSmem {
  float red[2][kAbWarps][kAbTileRows];
  float ssq[kAbWarps];
  float bias_a[kAbMaxRows];                 // q/k/v biases of rows [a0, a1)
  float bias_d[kAbMaxRows], resid[kAbMaxRows];  // o-proj bias and residual of rows [d0, d1)
  float q[kAbMaxRep][kAbHd];                // rotated q of the split's query heads
  float kn[kAbHd], vn[kAbHd];               // rotated new key, new value
  float sp[kAbMaxRep][kAbKeyBlock];         // probabilities of the current key block
  uint64_t full[kAbStages], empty[kAbStages];
  int issued;
  int prod_done;
  int ok;
  int last;  // this CTA merges its kv head's splits
};

template <int NCH_A, int NCH_D>
__global__ void __launch_bounds__(kAbThreads, 1) attn_block_kernel(const __grid_constant__ AbArgs a) {
  extern __shared__ __align__(128) uint8_t ab_smem[];
  uint8_t* ring = ab_smem;
  AbSmem& S = *reinterpret_cast<AbSmem*>(ab_smem + kAbStages * kAbStageBytes);
  const ns_attn_block_t& p = a.p;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, c = blockIdx.x;
  const int H = p.H, hd = kAbHd, n_rep = p.n_head / p.n_head_kv;

  // the token's position (written before this step's kernels: chain invariant).  The load is issued
  // here and first waited for where the key split is planned, after the q/k/v rows are requested.
  const int pos_raw = *p.pos;

  if (tid == 0) {
    stamp(a.trace, kAbEvStart);
    S.issued = 0;
    S.prod_done = 0;
    S.ok = 1;
    for (int i = 0; i < kAbStages; ++i) {
      mbar_init(&S.full[i], 1);
      mbar_init(&S.empty[i], kAbWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kAbWarps) {
    // ================================================================= producer: the byte stream
    if (lane == 0) {
      const uint8_t* wseg[3] = {static_cast<const uint8_t*>(p.wq), static_cast<const uint8_t*>(p.wk),
                                static_cast<const uint8_t*>(p.wv)};
      const int seg0[4] = {0, a.qd, a.qd + a.kvd, a.qkv_rows};
      // the q/k/v tiles do not depend on the position: they go out first, the rest once it is known
      AbPlan pl = ab_plan(a, 0, c, G);
      int i = 0;
      bool stop = false;
      auto next_slot = [&](int i) -> int {
        const int slot = i % kAbStages;
        if (i >= kAbStages && !mbar_wait_bounded(&S.empty[slot], (uint32_t)((i / kAbStages - 1) & 1))) stop = true;
        return slot;
      };
      for (; i < pl.nA; ++i) {  // q/k/v rows (three matrices, one concatenated row space)
        const int slot = next_slot(i);
        if (stop) break;
        uint8_t* dst = ring + (size_t)slot * kAbStageBytes;
        const int r0 = pl.a0 + i * kAbTileRows, r1 = min(r0 + kAbTileRows, pl.a1);
        mbar_arrive_expect_tx(&S.full[slot], (uint32_t)((r1 - r0) * H * 2));
        for (int sg = 0; sg < 3; ++sg) {
          const int lo = max(r0, seg0[sg]), hi = min(r1, seg0[sg + 1]);
          if (lo < hi)
            ab_copy(dst + (size_t)(lo - r0) * H * 2, wseg[sg] + (int64_t)(lo - seg0[sg]) * H * 2,
                    (uint32_t)((hi - lo) * H * 2), &S.full[slot]);
        }
      }
      const int pos = pos_raw;
      if (!stop && pos >= 0 && pos < p.max_ctx) {
        pl = ab_plan(a, pos, c, G);
        const int64_t cache_g = (int64_t)pl.g * p.max_ctx * hd;
        for (int b = 0; b < pl.nB; ++b, ++i) {  // keys / values of one block (slots below pos only)
          const int slot = next_slot(i);
          if (stop) break;
          uint8_t* dst = ring + (size_t)slot * kAbStageBytes;
          const int kb = pl.j0 + b * kAbKeyBlock, ke = min(kb + kAbKeyBlock, pl.j1), kc = min(ke, pos);
          const uint32_t n = kc > kb ? (uint32_t)((kc - kb) * hd * 4) : 0u;
          mbar_arrive_expect_tx(&S.full[slot], 2 * n);
          if (n) {
            ab_copy(dst, reinterpret_cast<const uint8_t*>(p.k_cache + cache_g + (int64_t)kb * hd), n, &S.full[slot]);
            ab_copy(dst + kAbKeyBlock * hd * 4, reinterpret_cast<const uint8_t*>(p.v_cache + cache_g + (int64_t)kb * hd),
                    n, &S.full[slot]);
          }
        }
        const int kq = p.n_head * hd;
        for (int t = 0; t < pl.nD && !stop; ++t, ++i) {  // o-proj rows
          const int slot = next_slot(i);
          if (stop) break;
          uint8_t* dst = ring + (size_t)slot * kAbStageBytes;
          const int r0 = pl.d0 + t * kAbTileRows, r1 = min(r0 + kAbTileRows, pl.d1);
          mbar_arrive_expect_tx(&S.full[slot], (uint32_t)((r1 - r0) * kq * 2));
          ab_copy(dst, static_cast<const uint8_t*>(p.wo) + (int64_t)r0 * kq * 2, (uint32_t)((r1 - r0) * kq * 2),
                  &S.full[slot]);
        }
      }
      S.issued = i;
      __threadfence_block();
      *reinterpret_cast<volatile int*>(&S.prod_done) = 1;
    }
    return;
  }

  // ================================================================= compute warps
  volatile int* okp = &S.ok;
  int done = 0;  // stream tiles consumed
  auto wait_tile = [&](int i) -> bool {
    return mbar_wait_bounded(&S.full[i % kAbStages], (uint32_t)((i / kAbStages) & 1));
  };
  auto release_tile = [&](int i) {
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.empty[i % kAbStages]);
  };

  AbPlan pl = ab_plan(a, 0, c, G);  // the row ranges (the key split is planned once pos is known)
  griddep_wait();
  // ---- x, RMSNorm weight, staged epilogue data: every load issued before any is used
  float xv[NCH_A][8];
  {
    const int nchunk = H / 8;
    float wn[NCH_A][8];
#pragma unroll
    for (int cc = 0; cc < NCH_A; ++cc) {
      const int ch = tid + cc * kAbWarps * 32;
      const bool in = ch < nchunk;
      const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 lo = in ? reinterpret_cast<const float4*>(p.x)[2 * ch] : z;
      const float4 hi = in ? reinterpret_cast<const float4*>(p.x)[2 * ch + 1] : z;
      const float4 wl = in ? reinterpret_cast<const float4*>(p.norm_w)[2 * ch] : z;
      const float4 wh = in ? reinterpret_cast<const float4*>(p.norm_w)[2 * ch + 1] : z;
      xv[cc][0] = lo.x; xv[cc][1] = lo.y; xv[cc][2] = lo.z; xv[cc][3] = lo.w;
      xv[cc][4] = hi.x; xv[cc][5] = hi.y; xv[cc][6] = hi.z; xv[cc][7] = hi.w;
      wn[cc][0] = wl.x; wn[cc][1] = wl.y; wn[cc][2] = wl.z; wn[cc][3] = wl.w;
      wn[cc][4] = wh.x; wn[cc][5] = wh.y; wn[cc][6] = wh.z; wn[cc][7] = wh.w;
    }
    float ba = 0.f, bd = 0.f, rd = 0.f;  // one staged row each (a CTA owns < 256 rows of either)
    const int ia = tid, id = tid;
    if (ia < pl.a1 - pl.a0) {
      const int row = pl.a0 + ia;
      const float* b = row < a.qd ? p.bq : row < a.qd + a.kvd ? p.bk : p.bv;
      const int lr = row < a.qd ? row : row < a.qd + a.kvd ? row - a.qd : row - a.qd - a.kvd;
      ba = b ? b[lr] : 0.f;
    }
    if (id < pl.d1 - pl.d0) {
      bd = p.bo ? p.bo[pl.d0 + id] : 0.f;
      rd = p.x[pl.d0 + id];
    }
    float ss = 0.f;
#pragma unroll
    for (int cc = 0; cc < NCH_A; ++cc)
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(xv[cc][j], xv[cc][j], ss);
    if (ia < pl.a1 - pl.a0) S.bias_a[ia] = ba;
    if (id < pl.d1 - pl.d0) {
      S.bias_d[id] = bd;
      S.resid[id] = rd;
    }
    if (tid == 0 && !(pos_raw >= 0 && pos_raw < p.max_ctx)) {  // a position outside the cache: no work
      *okp = 0;
      if (c == 0) raise_device_error(NS_DEVERR_ROUTE);
    }
    ss = warp_sum(ss);
    if (lane == 0) S.ssq[warp] = ss;
    named_sync(1, kAbWarps * 32);
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kAbWarps; ++w) tot += S.ssq[w];
    const float r = 1.0f / sqrtf(tot / (float)H + p.rms_eps);
#pragma unroll
    for (int cc = 0; cc < NCH_A; ++cc)
#pragma unroll
      for (int j = 0; j < 8; ++j) xv[cc][j] = __fmul_rn(__fmul_rn(xv[cc][j], r), wn[cc][j]);  // (x * r) * w
  }
  griddep_launch_dependents();
  if (tid == 0) stamp(a.trace, kAbEvNorm);

  // ---- phase A: q, k, v rows of this CTA
  bool alive = *okp != 0;
  for (int i = 0; i < pl.nA && alive; ++i) {
    const bool landed = wait_tile(i);
    const int r0 = pl.a0 + i * kAbTileRows, rows = min(kAbTileRows, pl.a1 - r0);
    const float sum = ab_tile<NCH_A>(ring + (size_t)(i % kAbStages) * kAbStageBytes, H, rows, xv, &S.red[0][0][0],
                                     i & 1, tid, lane, warp);
    release_tile(i);
    if (tid < rows) a.yqkv[r0 + tid] = sum + S.bias_a[r0 - pl.a0 + tid];
    if (!landed) *okp = 0;
    done = i + 1;
    named_sync(1, kAbWarps * 32);
    alive = *okp != 0;
  }
  {  // every CTA arrives at every grid barrier, also after a failure of its own, so that no other
    // CTA waits for it until its limit
    if (tid == 0) stamp(a.trace, kAbEvPhaseA);
    const bool synced = ab_grid_sync(a.bar, G, tid, okp);
    alive = alive && synced;
    if (tid == 0) stamp(a.trace, kAbEvBar1);
  }

  // ---- phase B: this CTA's key split of one kv head
  const int pos = alive ? pos_raw : 0;
  pl = ab_plan(a, pos, c, G);
  if (alive && pl.item >= 0) {
    const float* cs = p.rope_cos + (int64_t)pos * hd;
    const float* sn = p.rope_sin + (int64_t)pos * hd;
    const int g = pl.g;
    for (int i = tid; i < n_rep * hd; i += kAbWarps * 32) {
      const int h = i / hd, d = i % hd;
      const float* qh = a.yqkv + (int64_t)(g * n_rep + h) * hd;
      const float rot = d < hd / 2 ? -__ldcg(qh + d + hd / 2) : __ldcg(qh + d - hd / 2);
      S.q[h][d] = __fadd_rn(__fmul_rn(__ldcg(qh + d), cs[d]), __fmul_rn(rot, sn[d]));
    }
    if (tid < hd) {
      const float* kh = a.yqkv + a.qd + (int64_t)g * hd;
      const float rot = tid < hd / 2 ? -__ldcg(kh + tid + hd / 2) : __ldcg(kh + tid - hd / 2);
      S.kn[tid] = __fadd_rn(__fmul_rn(__ldcg(kh + tid), cs[tid]), __fmul_rn(rot, sn[tid]));
      S.vn[tid] = __ldcg(a.yqkv + a.qd + a.kvd + (int64_t)g * hd + tid);
    }
    named_sync(1, kAbWarps * 32);
    if (pl.s == a.splits - 1 && tid < hd) {  // append the token's key and value to the cache
      const int64_t o = (int64_t)g * p.max_ctx * hd + (int64_t)pos * hd + tid;
      p.k_cache[o] = S.kn[tid];
      p.v_cache[o] = S.vn[tid];
    }
    const bool head_ok = warp < n_rep;
    float m = -INFINITY, l = 0.f, acc0 = 0.f, acc1 = 0.f;
    for (int b = 0; b < pl.nB; ++b) {
      const int i = pl.nA + b;
      const bool landed = wait_tile(i);
      uint8_t* st = ring + (size_t)(i % kAbStages) * kAbStageBytes;
      float* Kb = reinterpret_cast<float*>(st);
      float* Vb = reinterpret_cast<float*>(st + kAbKeyBlock * hd * 4);
      const int kb = pl.j0 + b * kAbKeyBlock, nb = min(kAbKeyBlock, pl.j1 - kb);
      if (pos >= kb && pos < kb + nb && tid < hd) {  // the token's own key/value (not in the cache copy)
        Kb[(pos - kb) * hd + tid] = S.kn[tid];
        Vb[(pos - kb) * hd + tid] = S.vn[tid];
      }
      named_sync(1, kAbWarps * 32);
      if (head_ok && landed) {
        float sc[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int j = lane + 32 * u;
          float dot = 0.f;
          if (j < nb) {
#pragma unroll
            for (int cc = 0; cc < hd / 4; ++cc) {
              const int col = ((cc + lane) & (hd / 4 - 1)) * 4;  // rotated: conflict-free 16-byte rows
              const float4 kv = *reinterpret_cast<const float4*>(Kb + j * hd + col);
              const float4 qv = *reinterpret_cast<const float4*>(&S.q[warp][col]);
              dot = fmaf(qv.x, kv.x, dot);
              dot = fmaf(qv.y, kv.y, dot);
              dot = fmaf(qv.z, kv.z, dot);
              dot = fmaf(qv.w, kv.w, dot);
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
        const float corr = expf(m - m_new);
        const float p0 = expf(sc[0] - m_new), p1 = expf(sc[1] - m_new);
        S.sp[warp][lane] = p0;
        S.sp[warp][lane + 32] = p1;
        l = l * corr + warp_sum(p0 + p1);
        acc0 *= corr;
        acc1 *= corr;
        m = m_new;
        __syncwarp();
        for (int j = 0; j < nb; ++j) {
          const float pj = S.sp[warp][j];
          const float2 vv = *reinterpret_cast<const float2*>(Vb + j * hd + 2 * lane);
          acc0 = fmaf(pj, vv.x, acc0);
          acc1 = fmaf(pj, vv.y, acc1);
        }
      }
      release_tile(i);
      if (!landed) *okp = 0;
      done = i + 1;
      named_sync(1, kAbWarps * 32);
    }
    if (head_ok) {
      float* ph = a.part + (((int64_t)g * a.splits + pl.s) * kAbMaxRep + warp) * kAbPartStride;
      if (lane == 0) {
        ph[0] = m;
        ph[1] = l;
      }
      ph[2 + 2 * lane] = acc0;
      ph[3 + 2 * lane] = acc1;
    }
    // the last split of kv head g to finish merges all of them (no grid barrier for the merge)
    named_sync(1, kAbWarps * 32);
    if (tid == 0) {
      __threadfence();
      S.last = atom_add_acq_rel(a.cnt + g, 1u) == (unsigned)(a.splits - 1);
    }
    named_sync(1, kAbWarps * 32);
    if (S.last) {
      __threadfence();
      if (head_ok) {
        // the splits' records, 16 at a time with all loads of a group in flight, merged with a
        // running maximum in split order, together with the head's sink
        const int h = g * n_rep + warp;
        const float* base = a.part + ((int64_t)g * a.splits * kAbMaxRep + warp) * kAbPartStride;
        constexpr int kGrp = 16;
        float mt = p.sinks ? p.sinks[h] : -INFINITY;
        float lt = p.sinks ? 1.0f : 0.f, o0 = 0.f, o1 = 0.f;  // relative to mt
        for (int t0 = 0; t0 < a.splits; t0 += kGrp) {
          float ms[kGrp], ls[kGrp], x0[kGrp], x1[kGrp];
#pragma unroll
          for (int u = 0; u < kGrp; ++u) {
            const int t = t0 + u;
            const float* q = base + (int64_t)t * kAbMaxRep * kAbPartStride;
            const bool in = t < a.splits;
            ms[u] = in ? __ldcg(q) : -INFINITY;
            ls[u] = in ? __ldcg(q + 1) : 0.f;
            x0[u] = in ? __ldcg(q + 2 + 2 * lane) : 0.f;
            x1[u] = in ? __ldcg(q + 3 + 2 * lane) : 0.f;
          }
          float mg = mt;
#pragma unroll
          for (int u = 0; u < kGrp; ++u) mg = fmaxf(mg, ms[u]);
          if (mg != mt) {  // rescale what was merged so far to the new maximum
            const float f = mt == -INFINITY ? 0.f : expf(mt - mg);
            lt *= f;
            o0 *= f;
            o1 *= f;
            mt = mg;
          }
#pragma unroll
          for (int u = 0; u < kGrp; ++u)
            if (ms[u] != -INFINITY) {  // a split with no keys adds nothing
              const float f = expf(ms[u] - mt);
              lt = fmaf(ls[u], f, lt);
              o0 = fmaf(x0[u], f, o0);
              o1 = fmaf(x1[u], f, o1);
            }
        }
        a.attn[(int64_t)h * hd + 2 * lane] = o0 / lt;
        a.attn[(int64_t)h * hd + 2 * lane + 1] = o1 / lt;
      }
      if (tid == 0) a.cnt[g] = 0u;  // ready for the next launch (stream-ordered)
    }
    alive = *okp != 0;
  }
  {
    if (tid == 0) stamp(a.trace, kAbEvPhaseB);
    const bool synced = ab_grid_sync(a.bar, G, tid, okp);
    alive = alive && synced;
    if (tid == 0) stamp(a.trace, kAbEvBar2);
  }

  // ---- phase D: o-proj rows of this CTA, + bias, + residual
  if (alive) {
    const int K = p.n_head * hd, nchunk = K / 8;
    float av[NCH_D][8];
#pragma unroll
    for (int cc = 0; cc < NCH_D; ++cc) {
      const int ch = tid + cc * kAbWarps * 32;
#pragma unroll
      for (int j = 0; j < 8; ++j) av[cc][j] = ch < nchunk ? __ldcg(a.attn + 8 * ch + j) : 0.f;
    }
    for (int t = 0; t < pl.nD && alive; ++t) {
      const int i = pl.nA + pl.nB + t;
      const bool landed = wait_tile(i);
      const int r0 = pl.d0 + t * kAbTileRows, rows = min(kAbTileRows, pl.d1 - r0);
      const float sum = ab_tile<NCH_D>(ring + (size_t)(i % kAbStages) * kAbStageBytes, K, rows, av, &S.red[0][0][0],
                                       i & 1, tid, lane, warp);
      release_tile(i);
      if (tid < rows) {
        const int li = r0 - pl.d0 + tid;
        p.out[r0 + tid] = S.resid[li] + (sum + S.bias_d[li]);
      }
      if (!landed) *okp = 0;
      done = i + 1;
      named_sync(1, kAbWarps * 32);
      alive = *okp != 0;
    }
  }

  if (tid == 0) stamp(a.trace, kAbEvEnd);
  if (!alive && tid == 0) {
    // let the copies still in flight land before the CTA's shared memory goes away (bounded waits)
    raise_device_error(NS_DEVERR_COPY_WAIT);
    const uint64_t t0 = globaltimer_ns();
    while (!*reinterpret_cast<volatile int*>(&S.prod_done) && globaltimer_ns() - t0 < 2 * kWaitLimitNs) __nanosleep(256);
    if (*reinterpret_cast<volatile int*>(&S.prod_done))
      for (int j = done; j < S.issued; ++j) (void)mbar_wait_bounded(&S.full[j % kAbStages], (uint32_t)((j / kAbStages) & 1));
  }
}

static int ab_check(const ns_attn_block_t* p, int nsm, int* splits) {
  if (!p) return fail(NS_ERR_INVALID, "ns_attn_block: null parameters");
  if (p->head_dim != kAbHd) return fail(NS_ERR_UNSUPPORTED, "ns_attn_block: head_dim %d (only 64)", p->head_dim);
  if (p->n_head_kv < 1 || p->n_head % p->n_head_kv || p->n_head / p->n_head_kv > kAbMaxRep)
    return fail(NS_ERR_UNSUPPORTED, "ns_attn_block: %d query heads over %d kv heads", p->n_head, p->n_head_kv);
  if (p->H < 8 || p->H % 8 || 8 * p->H * 2 > kAbStageBytes || 8 * p->n_head * kAbHd * 2 > kAbStageBytes)
    return fail(NS_ERR_UNSUPPORTED, "ns_attn_block: H=%d, n_head=%d outside the stage size", p->H, p->n_head);
  if (p->max_ctx < 1 || p->window < 0) return fail(NS_ERR_INVALID, "ns_attn_block: bad max_ctx / window");
  if (p->n_head_kv > 48) return fail(NS_ERR_UNSUPPORTED, "ns_attn_block: more than 48 kv heads");
  const int qkv = p->n_head * kAbHd + 2 * p->n_head_kv * kAbHd;
  if ((qkv + nsm - 1) / nsm > kAbMaxRows || (p->H + nsm - 1) / nsm > kAbMaxRows)
    return fail(NS_ERR_UNSUPPORTED, "ns_attn_block: more than %d rows per SM", kAbMaxRows);
  const int keys = p->window > 0 ? std::min(p->window + 1, p->max_ctx) : p->max_ctx;
  *splits = std::max(1, std::min(nsm / p->n_head_kv, (keys + kAbKeyBlock - 1) / kAbKeyBlock));
  return NS_OK;
}

static size_t ab_ws_layout(const ns_attn_block_t* p, int splits, size_t* off_y, size_t* off_part, size_t* off_attn) {
  size_t off = 256;  // barrier counter at 0, per-kv-head split counters at 64
  *off_y = off;
  off += align_up((size_t)(p->n_head + 2 * p->n_head_kv) * kAbHd * 4, 256);
  *off_part = off;
  off += align_up((size_t)p->n_head_kv * splits * kAbMaxRep * kAbPartStride * 4, 256);
  *off_attn = off;
  off += align_up((size_t)p->n_head * kAbHd * 4, 256);
  return off;
}

template <int NA, int ND>
static int launch_ab(const AbArgs& a, int grid, cudaStream_t s) {
  auto kern = attn_block_kernel<NA, ND>;
  const size_t smem = (size_t)kAbStages * kAbStageBytes + sizeof(AbSmem);
  NS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int per_sm = 0;
  NS_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kAbThreads, smem));
  if (per_sm < 1) return fail(NS_ERR_UNSUPPORTED, "ns_attn_block: kernel does not fit on an SM");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kAbThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  NS_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a));
  return NS_OK;
}

}  // namespace ns

extern "C" int ns_attn_block_workspace_bytes(const ns_attn_block_t* p, size_t* bytes) {
  using namespace ns;
  if (!bytes) return fail(NS_ERR_INVALID, "ns_attn_block_workspace_bytes: null output");
  int nsm = 0, splits = 0;
  int st = num_sms(&nsm);
  if (!st) st = ab_check(p, nsm, &splits);
  if (st) return st;
  size_t oy, op, oa;
  *bytes = ab_ws_layout(p, splits, &oy, &op, &oa);
  return NS_OK;
}

extern "C" int ns_attn_block(const ns_attn_block_t* p, void* workspace, size_t workspace_bytes, ns_stream_t stream) {
  using namespace ns;
  int nsm = 0, splits = 0;
  int st = num_sms(&nsm);
  if (!st) st = ab_check(p, nsm, &splits);
  if (st) return st;
  size_t oy, op, oa;
  const size_t need = ab_ws_layout(p, splits, &oy, &op, &oa);
  if (!workspace || workspace_bytes < need)
    return fail(NS_ERR_SIZE, "ns_attn_block: workspace of %zu bytes, need %zu", workspace_bytes, need);
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return fail(NS_ERR_INVALID, "ns_attn_block: workspace not 256-byte aligned");
  if (!p->x || !p->norm_w || !p->wq || !p->wk || !p->wv || !p->wo || !p->pos || !p->rope_cos || !p->rope_sin ||
      !p->k_cache || !p->v_cache || !p->out)
    return fail(NS_ERR_INVALID, "ns_attn_block: null pointer");
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  if (!al16(p->x) || !al16(p->norm_w) || !al16(p->wq) || !al16(p->wk) || !al16(p->wv) || !al16(p->wo) ||
      !al16(p->k_cache) || !al16(p->v_cache))
    return fail(NS_ERR_INVALID, "ns_attn_block: x, norm_w, weights and caches must be 16-byte aligned");
  AbArgs a;
  memset(&a, 0, sizeof a);
  a.p = *p;
  a.qd = p->n_head * kAbHd;
  a.kvd = p->n_head_kv * kAbHd;
  a.qkv_rows = a.qd + 2 * a.kvd;
  a.splits = splits;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  a.bar = reinterpret_cast<unsigned long long*>(ws);
  a.yqkv = reinterpret_cast<float*>(ws + oy);
  a.part = reinterpret_cast<float*>(ws + op);
  a.attn = reinterpret_cast<float*>(ws + oa);
  a.cnt = reinterpret_cast<unsigned*>(ws + 64);
  a.trace = g_trace_buf[trace_slot()];
  const int na = (p->H / 8 + kAbWarps * 32 - 1) / (kAbWarps * 32), nd = (a.qd / 8 + kAbWarps * 32 - 1) / (kAbWarps * 32);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (na == 1 && nd == 1) return launch_ab<1, 1>(a, nsm, s);
  if (na == 1 && nd == 2) return launch_ab<1, 2>(a, nsm, s);
  if (na == 2 && nd == 2) return launch_ab<2, 2>(a, nsm, s);
  if (na == 2 && nd == 1) return launch_ab<2, 1>(a, nsm, s);
  return fail(NS_ERR_UNSUPPORTED, "ns_attn_block: H=%d / %d query heads beyond 4096 columns", p->H, p->n_head);
}
