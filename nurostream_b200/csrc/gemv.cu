// ns_gemv: fused dequant-GEMV from GGUF bytes (batch 1..NS_MAX_TOKENS).
//
// Layout: each CTA owns a contiguous run of rows, walked in tiles of TILE rows
// (16, or 8 for wide rows and several tokens).  A tile's bytes are one
// contiguous range of the weight buffer; thread 0 streams tiles into a ring of
// shared-memory stages with 1-D bulk copies (the TMA engine, completion on an
// mbarrier).  The activations are converted to fp32 once per CTA and kept in
// shared memory, each 32-element group padded to kXG floats so that lanes
// reading different groups hit different banks.
//
// Q8_0 and Q4_K take their weights as the int8 / 4-bit integers they are and
// the activations as three int8 digit planes per 32-element group (an exact
// 22-bit fixed point of the group, scale 2^(e-22) with max|x| < 2^e): the
// group's dot product is three dp4a chains per weight word, combined in fp32
// and scaled once.  MXFP4 and Q6_K decode to fp32 and use fp32 FMAs (an
// MXFP4 variant on dp4a, with the e2m1 nibbles mapped to int8 by prmt table
// lookups, measured slower: the decode costs as much as the conversions).
//
// Work split of a tile: the W warps take interleaved slices of K, and each
// warp's lanes form RS row subsets of LG = 32/RS lanes: lane (s, j) takes the
// R = TILE/RS rows sR .. sR + R - 1 of the tile and the groups w*LG + j,
// + W*LG, .. of K.  So every lane runs R independent row sums and loads each
// activation group once for all of them.  The rows of a subset are one
// "piece" of the stage: when rows start on 16-byte boundaries each piece is
// one bulk copy into a slot whose pitch keeps the subsets on different banks.  Lane sums meet by shuffles within each subset,
// then across the W warps in shared memory, in a fixed order.  One token:
// 16 warps x 4 subsets (4 rows a lane); more tokens: 8 warps x 2 subsets.
#include "qdot.cuh"

namespace ns {

constexpr int kGemvMaxWarps = 16;
constexpr int kGemvMaxStages = 6;
constexpr int kGemvEarlyTiles = 1;  // tiles requested before the activations are staged
constexpr int kSmemBudget = 220 * 1024;
constexpr int kXG = 36;     // shared-memory floats per 32-element group of x (fp32 path)

template <int FMT>
struct GemvInt8 {
  static constexpr bool value = FMT == NS_GGML_Q8_0 || FMT == NS_GGML_Q4_K;
};

// Shared-memory bytes of the activations of NT token slots (K elements each).
__host__ __device__ inline size_t gemv_x_bytes(bool int8, int nt, int K) {
  const size_t ng = (size_t)K / 32;
  return int8 ? (size_t)nt * ng * (kXQG + 8) : (size_t)nt * ng * kXG * 4;
}

// Integer-path dot products: rows[r] (shared memory) against token slots t of the activation
// planes xq (plane p of group g at xq + t*xqs + g*kXQG + 32p), with per-group scales xsc and
// sums xsum (at t*ng + g).
template <int FMT, int NT, int R>
__device__ __forceinline__ void dot_rows_i8(const uint8_t* const (&rows)[R], int ngroups, int g0, int gstep,
                                            const uint8_t* xq, int xqs, const float* xsc, const float* xsum,
                                            float (&acc)[R][NT], bool rows16) {
  for (int g = g0; g < ngroups; g += gstep) {
    uint32_t q[R][8];
    float da[R], db[R];  // Q8_0: d, 0; Q4_K: d*sc, dmin*mn
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (FMT == NS_GGML_Q8_0) {
        uint32_t w[9];
        lds_words_unaligned<9>(rows[r] + 34 * g, w);
        da[r] = f16_bits_to_float(w[0]);
        db[r] = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) q[r][i] = __funnelshift_r(w[i], w[i + 1], 16);  // signed int8 x 4
      } else {
        QGroup<NS_GGML_Q4_K> qg;
        if (rows16)  // rows start on 16-byte boundaries
          qg.load_aligned(rows[r], g);
        else
          qg.load(rows[r], g);
        da[r] = qg.dsc;
        db[r] = qg.mmn;
#pragma unroll
        for (int i = 0; i < 8; ++i) q[r][i] = qg.q[i];  // 0..15 x 4
      }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const uint4* xp = reinterpret_cast<const uint4*>(xq + (size_t)t * xqs + (size_t)g * kXQG);
      uint32_t xw[3][8];
#pragma unroll
      for (int p = 0; p < 3; ++p) {
        const uint4 lo = xp[2 * p], hi = xp[2 * p + 1];
        xw[p][0] = lo.x; xw[p][1] = lo.y; xw[p][2] = lo.z; xw[p][3] = lo.w;
        xw[p][4] = hi.x; xw[p][5] = hi.y; xw[p][6] = hi.z; xw[p][7] = hi.w;
      }
      const float sc = xsc[t * ngroups + g], sm = xsum[t * ngroups + g];
#pragma unroll
      for (int r = 0; r < R; ++r) {
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
}

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
  int stages;
  int stage_bytes;
  int pitch;  // shared-memory bytes between pieces of R rows: R*rb, or more (padded piece copies)
};

template <int FMT, int NT, int TILE, int W, int RS>
__global__ void __launch_bounds__((W + 1) * 32, 1) gemv_kernel(GemvArgs a) {
  // W compute warps (kThreads threads) and one producer warp, warp W
  constexpr int kThreads = W * 32, LG = 32 / RS, R = TILE / RS;  // lanes per row subset, rows per lane
  static_assert(32 % W == 0 && (TILE * NT) % (32 / W) == 0, "final reduce: whole warps per pass");
  extern __shared__ __align__(128) uint8_t smem[];
  const int K = a.K, T = a.T, nst = a.stages;
  constexpr bool kInt = GemvInt8<FMT>::value;
  const int ngroups = K / 32;
  float* xs = reinterpret_cast<float*>(smem);               // fp32 path: padded groups
  const int xt = ngroups * kXG;                             // floats per token
  uint8_t* xq = smem;                                       // integer path: digit planes
  const int xqs = ngroups * kXQG;                           // bytes per token
  float* xsc = reinterpret_cast<float*>(smem + (size_t)NT * xqs);  // [token][group] scale 2^(e-22)
  float* xsum = xsc + NT * ngroups;                         // [token][group] sum of x
  float* red = reinterpret_cast<float*>(smem + gemv_x_bytes(kInt, NT, K));  // 2 x [warp][row][token]
  uint8_t* stages = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(red + 2 * W * TILE * NT) + 127) & ~uintptr_t(127));
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + nst * a.stage_bytes);  // stage landed
  uint64_t* empty = full + nst;                                                 // stage consumed

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  // contiguous, balanced row range of this CTA
  const int r_begin = (int)((int64_t)a.n_rows * blockIdx.x / gridDim.x);
  const int r_end = (int)((int64_t)a.n_rows * (blockIdx.x + 1) / gridDim.x);
  const int n_tiles = (r_end - r_begin + TILE - 1) / TILE;

  auto tile_span = [&](int i) -> Span {
    int r0 = r_begin + i * TILE;
    int r1 = min(r0 + TILE, r_end);
    return Span{a.w + (int64_t)r0 * a.rb, a.w + (int64_t)r1 * a.rb};
  };
  const bool row_copies = a.pitch != R * a.rb;  // rows 16-byte aligned: one copy per piece, padded slots
  auto issue = [&](int i) {
    uint64_t* bar = &full[i % nst];
    uint8_t* dst = stages + (i % nst) * a.stage_bytes;
    Span s = tile_span(i);
    if (row_copies) {
      const int nr = (int)((s.g1 - s.g0) / a.rb);
      mbar_arrive_expect_tx(bar, (uint32_t)(nr * a.rb));
      for (int p = 0; p * R < nr; ++p)
        bulk_g2s(dst + p * a.pitch, s.g0 + (int64_t)p * R * a.rb, (uint32_t)(min(R, nr - p * R) * a.rb), bar);
      return;
    }
    uintptr_t lo, hi;
    bulk_window(s, a.w, a.w_end, &lo, &hi);
    mbar_arrive_expect_tx(bar, hi > lo ? (uint32_t)(hi - lo) : 0u);
    issue_span_pieces(dst, s, a.w, a.w_end, bar, 4096u);
  };


  // The producer warp issues every copy: a bulk copy's issue blocks for a while once the SM's
  // copy queue is busy, which would otherwise stall a compute warp.  The first stages go out
  // before the activations are staged; the rest once x is in shared memory, since with every
  // SM's whole ring in flight the activation loads queue behind the weight stream.
  const int early = min(min(kGemvEarlyTiles, nst), n_tiles);
  if (warp == W) {
    if (lane == 0) {
      for (int s = 0; s < nst; ++s) {
        mbar_init(&full[s], 1);
        mbar_init(&empty[s], 1);
      }
      fence_mbar_init();
      for (int i = 0; i < early; ++i) issue(i);
    }
    __syncthreads();  // barriers initialised, x staged
    if (lane == 0) {
      for (int i = early; i < n_tiles; ++i) {
        if (i >= nst && !mbar_wait_bounded(&empty[i % nst], (uint32_t)((i / nst - 1) & 1))) break;
        issue(i);
      }
    }
    return;
  }
  // activations -> shared memory (overlaps with the first copies); token slots T..NT-1 hold zeros,
  // so every lane computes all NT slots without tests
  if (kInt) {
    // one thread per (token, group): balanced radix-256 digits of X = rint(x * 2^(22-e)),
    // |X| <= 2^22 with max|x| < 2^e, so every digit fits int8
    const bool x_vec = a.x_dtype == NS_F32 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 && (a.x_stride & 3) == 0;
    for (int it = tid; it < NT * ngroups; it += kThreads) {
      const int t = it / ngroups, g = it - t * ngroups;
      float v[32];
      if (t >= T) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.f;
      } else if (x_vec) {
        const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(a.x) + (int64_t)t * a.x_stride + 32 * g);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 f = src[j];
          v[4 * j] = f.x; v[4 * j + 1] = f.y; v[4 * j + 2] = f.z; v[4 * j + 3] = f.w;
        }
      } else {
        load_floats<32>(a.x, a.x_dtype, [&](int j) -> int64_t { return (int64_t)t * a.x_stride + 32 * g + j; }, v);
      }
      group_planes_i8(v, xq + (size_t)t * xqs + (size_t)g * kXQG, &xsc[t * ngroups + g], &xsum[t * ngroups + g]);
    }
  } else if (a.x_dtype == NS_F32 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 && (a.x_stride & 3) == 0) {
    // fp32 x: 4 elements a load (a group's padded row is 144 B, so float4 stores stay aligned)
    constexpr int kB = 4;
    const int n4 = NT * K / 4;
    for (int i0 = tid; i0 < n4; i0 += kB * kThreads) {
      float4 vb[kB];
#pragma unroll
      for (int b = 0; b < kB; ++b) {
        const int i = i0 + b * kThreads, t = 4 * i / K, k = 4 * i - t * K;
        vb[b] = i < n4 && t < T ? *reinterpret_cast<const float4*>(static_cast<const float*>(a.x) + (int64_t)t * a.x_stride + k)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int b = 0; b < kB; ++b) {
        const int i = i0 + b * kThreads, t = 4 * i / K, k = 4 * i - t * K;
        if (i < n4) *reinterpret_cast<float4*>(xs + t * xt + (k >> 5) * kXG + (k & 31)) = vb[b];
      }
    }
  } else {
    constexpr int kB = 8;  // elements per thread whose loads are issued together
    for (int i0 = tid; i0 < NT * K; i0 += kB * kThreads) {
      float vb[kB];
      load_floats<kB>(a.x, a.x_dtype, [&](int b) -> int64_t {
        const int i = i0 + b * kThreads, t = i / K, k = i - t * K;
        return i < NT * K && t < T ? (int64_t)t * a.x_stride + k : -1;
      }, vb);
#pragma unroll
      for (int b = 0; b < kB; ++b) {
        const int i = i0 + b * kThreads, t = i / K, k = i - t * K;
        if (i < NT * K) xs[t * xt + (k >> 5) * kXG + (k & 31)] = vb[b];
      }
    }
  }
  __syncthreads();

  const int sub = lane / LG, lg = lane % LG;
  int tok[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) tok[t] = t;
  for (int i = 0; i < n_tiles; ++i) {
    const int st = i % nst;
    uint8_t* buf = stages + st * a.stage_bytes;
    const Span s = tile_span(i);
    const bool ok = mbar_wait_bounded(&full[st], (uint32_t)((i / nst) & 1));
    if (!row_copies && span_has_ragged(s, a.w, a.w_end)) {
      if (warp == 0) copy_ragged(buf, s, a.w, a.w_end, lane);
      named_sync(1, kThreads);
    }
    const int r0 = r_begin + i * TILE;
    const int nr = (int)((s.g1 - s.g0) / a.rb);
    float* rd = red + (i & 1) * (W * TILE * NT);
    if (ok) {
      const uint8_t* base = row_copies ? buf : buf + (reinterpret_cast<uintptr_t>(s.g0) & 15);
      // this subset's rows sub, sub + RS, ..; those at or past nr repeat row nr - 1 and are dropped
      const uint8_t* rows[R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int q = min(sub * R + r, nr - 1);
        rows[r] = base + (q / R) * a.pitch + (q % R) * a.rb;
      }
      float acc[R][NT];
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;
      if constexpr (kInt)
        dot_rows_i8<FMT, NT, R>(rows, ngroups, warp * LG + lg, W * LG, xq, xqs, xsc, xsum, acc,
                                row_copies || ((reinterpret_cast<uintptr_t>(base) & 15) == 0 && a.rb % 16 == 0));
      else
        dot_rows<FMT, NT, R, kXG, true>(rows, R, ngroups, warp * LG + lg, xs, xt, tok, NT, acc, W * LG);
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          float v = acc[r][t];
#pragma unroll
          for (int o = 1; o < LG; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
          if (lg == 0) rd[(warp * TILE + sub * R + r) * NT + t] = v;
        }
    }
    named_sync(1, kThreads);  // stage st consumed, this tile's partial sums in rd
    if (tid == 0) mbar_arrive(&empty[st]);
    // the W warps' partials of each (row, token) meet in W consecutive lanes by shuffles, so no
    // thread runs a long serial sum that would hold up the next tile
    if (ok) {
      const int w = tid % W;
      for (int q = tid / W; q < TILE * NT; q += kThreads / W) {
        const int row = q / NT, t = q - row * NT;
        float v = rd[(w * TILE + row) * NT + t];
#pragma unroll
        for (int o = 1; o < W; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (w == 0 && row < nr && t < T) store_float(a.y, a.y_dtype, (int64_t)t * a.y_stride + r0 + row, v);
      }
    }
  }
}

template <int FMT, int NT, int TILE, int W, int RS>
static int launch_gemv(const GemvArgs& a, int grid, size_t smem, cudaStream_t stream) {
  auto kern = gemv_kernel<FMT, NT, TILE, W, RS>;
  // the kernel's whole budget, not this launch's size (see dense.cu: graphs replay against the attribute)
  NS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)std::max(smem, (size_t)kSmemBudget)));
  kern<<<grid, (W + 1) * 32, smem, stream>>>(a);
  NS_CUDA_TRY(cudaGetLastError());
  return NS_OK;
}

template <int FMT>
static int dispatch_gemv_t(const GemvArgs& a, int tile, int grid, size_t smem, cudaStream_t stream) {
  if (a.T == 1)
    return tile == 16 ? launch_gemv<FMT, 1, 16, 16, 4>(a, grid, smem, stream) : launch_gemv<FMT, 1, 8, 16, 4>(a, grid, smem, stream);
  if (a.T == 2) return launch_gemv<FMT, 2, 8, 8, 2>(a, grid, smem, stream);
  if (a.T <= 4) return launch_gemv<FMT, 4, 8, 8, 2>(a, grid, smem, stream);
  return launch_gemv<FMT, 8, 8, 8, 2>(a, grid, smem, stream);
}

}  // namespace ns

extern "C" int ns_gemv(const uint8_t* w, size_t w_bytes, int ggml_type, int n_rows, int K, const void* x,
                       int x_dtype, int64_t x_stride, int T, void* y, int y_dtype, int64_t y_stride,
                       ns_stream_t stream) {
  using namespace ns;
  if (ggml_type != NS_GGML_MXFP4 && ggml_type != NS_GGML_Q8_0 && ggml_type != NS_GGML_Q4_K &&
      ggml_type != NS_GGML_Q6_K && ggml_type != NS_GGML_Q5_K && ggml_type != NS_GGML_Q4_0)
    return fail(NS_ERR_UNSUPPORTED, "ns_gemv: ggml type %d has no fused GEMV (MXFP4, Q8_0, Q4_K, Q5_K, Q6_K, Q4_0)",
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
  // tiles of 16 rows for one token when they fit a stage of <= 48 KB, else 8
  const int tile = (T == 1 && 16 * rb + 32 <= 48 * 1024) ? 16 : 8;
  const int nt_slots = T == 1 ? 1 : T <= 2 ? 2 : T <= 4 ? 4 : 8;  // the kernel's NT
  const bool int8_path = ggml_type == NS_GGML_Q8_0 || ggml_type == NS_GGML_Q4_K;
  const size_t x_bytes = gemv_x_bytes(int8_path, nt_slots, K);
  const size_t red_bytes = (size_t)2 * (T == 1 ? 16 : 8) * tile * nt_slots * 4;
  // When rows start on 16-byte boundaries, each piece of R rows is one bulk copy into a slot
  // whose pitch is R*rb rounded up to a residue mod 128 B at which the lanes of a warp (subset
  // s reading row sR + r, blocks g..) spread over the 32 banks: at most 2-way conflicts,
  // against 4-way when rb is a multiple of 128.  Other rows are copied as one span.
  const int rs = T == 1 ? 4 : 2, rpp = tile / rs;
  const int residue = rs == 2 ? 64 : ggml_type == NS_GGML_MXFP4 ? 32 : 48;
  const bool rows_aligned = rb % 16 == 0 && reinterpret_cast<uintptr_t>(w) % 16 == 0;
  const int64_t pb = rpp * rb;
  const int pitch = (int)(rows_aligned ? pb + ((residue - pb % 128) + 128) % 128 : pb);
  const int stage_bytes = rows_aligned ? rs * pitch : (int)((tile * rb + 32 + 15) & ~int64_t(15));
  const size_t fixed = x_bytes + red_bytes + 128 + 2 * kGemvMaxStages * 8;
  const int stages = (int)std::min<size_t>(kGemvMaxStages, fixed < (size_t)kSmemBudget ? (kSmemBudget - fixed) / stage_bytes : 0);
  if (stages < 2)
    return fail(NS_ERR_UNSUPPORTED, "ns_gemv: T*K=%d activations plus two %d-row tiles of %lld-byte rows exceed shared memory",
                T * K, tile, (long long)rb);
  const int grid = std::min(nsm, n_rows);
  const size_t smem = fixed + (size_t)stages * stage_bytes;

  GemvArgs a{w, w + w_bytes, n_rows, K, (int)rb, T, x, x_dtype, x_stride, y, y_dtype, y_stride, stages, stage_bytes, pitch};
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (ggml_type) {
    case NS_GGML_MXFP4: return dispatch_gemv_t<NS_GGML_MXFP4>(a, tile, grid, smem, s);
    case NS_GGML_Q8_0: return dispatch_gemv_t<NS_GGML_Q8_0>(a, tile, grid, smem, s);
    case NS_GGML_Q4_K: return dispatch_gemv_t<NS_GGML_Q4_K>(a, tile, grid, smem, s);
    case NS_GGML_Q5_K: return dispatch_gemv_t<NS_GGML_Q5_K>(a, tile, grid, smem, s);
    case NS_GGML_Q4_0: return dispatch_gemv_t<NS_GGML_Q4_0>(a, tile, grid, smem, s);
    default: return dispatch_gemv_t<NS_GGML_Q6_K>(a, tile, grid, smem, s);
  }
}
