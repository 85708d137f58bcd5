// Fused MoE decode layer on the tcgen05 tensor cores (MXFP4 experts, T <= 2).
//
// Same contract and results (to fp32 rounding) as moe_layer_kernel in moe.cu;
// ns_moe_decode_layer picks this kernel when the layer qualifies
// (moe_tc_eligible).  One launch, one CTA per SM, every CTA resident at once.
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
// Staging.  A K-chunk of a tile is 14 blocks (238 bytes) of 128 rows.  Rows
// r, r+8, .. of one tile share their alignment (8 GGUF rows of a 64-multiple
// width are a 16-byte multiple), so one TMA box of 256 bytes x 16 row groups
// fetches row phase j of the chunk; 8 boxes (4 KB each) fill a stage.  Repack
// warps move each 17-byte block into the operand layout.
//
// Work.  A phase-1 tile is 128 neurons of one routed expert; its K runs over
// the gate rows and then the up rows (separate accumulators), so the
// activation of a neuron sees both in one thread.  A phase-2 tile is 128 down
// rows of one (token, expert) pair.  Each phase's K blocks are split evenly
// over the CTAs at chunk boundaries ("stream-K"), so every SM streams the same
// number of weight bytes; a CTA streams its phase-1 share, then its phase-2
// share.  A tile split over CTAs is finished by the last one to arrive, in a
// fixed summation order, so results are deterministic.  Phase 2 of expert e
// starts as soon as all tiles of e are done (per-expert counters); the
// combine of a row block runs when all of its pairs are done.  No grid
// barrier follows the routing barrier.
//
// Operands that stay put.  Phase 1's B (the token's activation planes) and its
// scales are built once per launch in shared memory / TMEM.  Phase 2's B (a
// pair's SwiGLU activation planes, written to the workspace by the phase-1
// epilogues of every CTA) is copied in once per pair by a loader warp into
// one of two shared-memory buffers, as soon as the pair's phase-1 tiles are
// counted done, and its scales are copied into TMEM as its chunks first need
// them; the repack warps never wait on other CTAs, so they keep staging
// phase-2 weights while the activations are still being finished elsewhere.
//
// Warps: 0 producer (TMA), 1 MMA issuer, 12 repack warps (raw rows into the
// operand layout), 4 epilogue warps (TMEM -> registers, finish tiles), 1
// phase-2 image loader.  Every
// wait is bounded; a wait that runs out raises a device error bit, stops the
// CTA's pipeline, lets in-flight copies and MMAs land, frees TMEM and returns.

#include "tc.cuh"

namespace ns {

constexpr int kTcWarps = 19;
constexpr int kTcThreads = kTcWarps * 32;
constexpr int kTcRepackWarps = 12;
// Warp roles.  Warp w issues from SM sub-partition w % 4 and can reach TMEM lanes 32*(w % 4) ..
// +31.  Producer 0, MMA issuer 1; one epilogue warp and three repack warps per lane quadrant:
// epilogue 16, 13, 14, 15 (quadrants 0..3), repack {4, 8, 12}, {5, 9, 17}, {2, 6, 10}, {3, 7, 11};
// 18 loads the phase-2 activation images.
constexpr int kTcMmaWarp = 1, kTcProducerWarp = 0, kTcLoaderWarp = 18;
__device__ __forceinline__ int tc_epi_quadrant(int w) {
  return w == 16 ? 0 : w == 13 ? 1 : w == 14 ? 2 : w == 15 ? 3 : -1;
}
// Repack index 3*quadrant + (0..2), or -1.
__device__ __forceinline__ int tc_repack_index(int w) {
  if (w < 2 || w == 13 || w == 14 || w == 15 || w == 16 || w >= 18) return -1;
  const int q = w & 3;
  const int wi = w == 17 ? 2 : (w >> 2) - (q <= 1 ? 1 : 0);
  return 3 * q + wi;
}
// M-row (TMEM lane) m = 32q + i of a tile holds tile row 8G + j, G = 8*(q/2) + i%8,
// j = 2*(i/8) + q%2: the 32 rows a quadrant's repack warps read sit in distinct banks of the
// staged boxes (8 row groups 4 banks apart x 4 row phases a quarter-quad apart when 8 GGUF rows
// are an odd multiple of 2 mod 16 bytes, as for 2880-wide rows).
__device__ __forceinline__ int tc_row_of(int m) {
  const int q = m >> 5, i = m & 31;
  return 8 * (8 * (q >> 1) + (i & 7)) + 2 * (i >> 3) + (q & 1);
}
constexpr int kTcCanStages = 2;
// Raw (TMA) stages: enough bytes in flight to cover the load latency; one fewer for T = 2, whose
// resident activation planes take the room.
template <int NT>
struct TcRaw {
  static constexpr int kStages = NT == 1 ? 5 : 4;
};
constexpr int kTcChunk = 14;                         // K blocks (32 elements) per chunk
constexpr int kTcBoxW = 272;                         // TMA box row (bytes, 136 u16): >= 14*17 + 14; rows of
                                                     // a box land 68 words apart (4 banks)
constexpr int kTcBoxRows = 16;                       // row groups per box (8 for half tiles)
constexpr int kTcBoxBytes = kTcBoxW * kTcBoxRows;    // one row phase of a chunk
constexpr int kTcRawBytes = 8 * kTcBoxBytes;         // 8 row phases
constexpr int kTcDCols = 32;                         // D: gate planes at +0, up planes at +16
// TMEM columns: D buffers [0, 64); weight scales (SFA) [64, 96), 2 stages x 16; weights (A)
// [128, 256), 2 stages x 64 (14 blocks x 4 used); activation scales resident for a whole K (4
// columns per 4-block atom): phase 1 [256, 384), phase 2 (the current pair) [384, 512).
constexpr int kTcTmemSfa = 64, kTcTmemA = 128, kTcTmemAStage = 64, kTcTmemSfb1 = 256, kTcTmemSfb2 = 384;
constexpr int kTcB2Bufs = 2;                         // phase-2 activation images in shared memory
constexpr int kTcTmemCols = 512;
constexpr int kTcMaxSegs = 8;                        // tiles one CTA touches
constexpr int kTcMaxSplit = 24;                      // CTAs one tile is split over
constexpr int kTcMaxTiles = 1024;
constexpr int kTcWsHeader = 8192;                    // barrier word, counters
constexpr int kTcOffCnt = 1024, kTcOffReady = kTcOffCnt + 4 * kTcMaxTiles, kTcOffCnt2 = kTcOffReady + 4 * 128;
constexpr int kTcMaxRowTiles = (kTcWsHeader - kTcOffCnt2) / 4;
constexpr int kTcSmemBudget = 225 * 1024;
constexpr int kTcGridMax = 160;                      // SMs the workspace is sized for

struct MoeTcArgs {
  // 8-row groups x 8*row_bytes bytes; box 256 x 16 (full tiles) and 256 x 8 (half tiles)
  CUtensorMap tm_gate16, tm_gate8, tm_up16, tm_up8, tm_down16, tm_down8;
  ns_moe_layer_t p;
  int rb_h, rb_f, nb_h, nb_f;
  unsigned long long* bar;
  unsigned* cnt;     // per tile: segments finished
  unsigned* ready;   // per slot: phase-1 tiles finished
  unsigned* cnt2;    // per phase-2 row tile: pairs finished
  float* logits;     // T x E
  float* partial;    // per CTA: 2 phase-1 slots of 2*T*128 floats, then 2 phase-2 slots of 128
  int part_floats;   // floats per CTA: (2*T + 1) * 128
  uint8_t* actimg;   // per pair: planes [nb_f][8][16], then scale atoms [nb_f/4][8][16] (bytes
                     // 0..3 of row p: plane p's scales of the atom's 4 blocks)
  float* yp;         // per pair: H fp32
  int img_bytes;
  int zero_tiles;    // counters to clear per launch
  int off_raw, off_b1, off_sfb1, off_b2, off_xchg, off_bars, off_shared;
  int b2_stride;      // bytes per phase-2 image buffer: planes (nb_f * 128), then scale atoms
  int sfb1_atom;     // bytes between phase-1 scale atoms (128 * T)
  unsigned long long* trace;
};

// A segment: K blocks [k0, k1) of one tile.  A tile split over CTAs is finished by the CTA that
// holds its first chunk (k0 == 0): the tile ends that CTA's range, so it is the last to get there.
// Every other sharer meets the tile at the start of its range (k0 > 0) and only publishes.
struct TcSeg {
  int tile, k0, k1;
  int grp, sub;                // slot (phase 1) or pair (phase 2), and 128-row block within it
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
  int nsh;                     // sharers of the tile being finished, other than this CTA
  short sh_cta[kTcMaxSplit];   // ... in ascending order
  __align__(16) float scratch[NS_MAX_EXPERTS];
};

// Geometry: phase-1 tiles (slot-major, 128 neurons, K = gate nb_h blocks then up nb_h blocks),
// then phase-2 tiles (pair-major, 128 down rows, K = nb_f blocks).
struct TcGeom {
  int T1, T2, ns1, nr2, nb_h, nb_f, H, F;
  __device__ int len(int ph) const { return ph == 0 ? 2 * nb_h : nb_f; }
  // K blocks of the half that block kb belongs to, and the half's first block
  __device__ void half_of(int ph, int kb, int* h0, int* hl) const {
    if (ph == 0 && kb >= nb_h) { *h0 = nb_h; *hl = nb_h; }
    else { *h0 = 0; *hl = ph == 0 ? nb_h : nb_f; }
  }
  // nearest chunk start to tile-local block `off` (chunks restart at each half)
  __device__ int snap(int ph, int off) const {
    int h0, hl;
    half_of(ph, off, &h0, &hl);
    const int w = off - h0;
    return h0 + min(hl, ((w + kTcChunk / 2) / kTcChunk) * kTcChunk);
  }
  // chunks of a tile and the tile-local block each starts at (chunks restart at each half)
  __device__ int nchunks(int ph) const {
    return ph == 0 ? 2 * ((nb_h + kTcChunk - 1) / kTcChunk) : (nb_f + kTcChunk - 1) / kTcChunk;
  }
  __device__ int chunk_start(int ph, int q) const {
    const int c0 = (nb_h + kTcChunk - 1) / kTcChunk;
    return ph == 0 && q >= c0 ? nb_h + kTcChunk * (q - c0) : kTcChunk * q;
  }
  // Each phase's K blocks (tile-major) are split evenly over the G CTAs at chunk boundaries:
  // CTA jj streams [bnd(jj), bnd(jj+1)).
  __device__ int bnd(int ph, int jj, int G) const {
    const int L = len(ph), U = (ph == 0 ? T1 : T2) * L;
    if (jj <= 0) return 0;
    if (jj >= G) return U;
    const int u = (int)(((unsigned)U * (unsigned)jj) / (unsigned)G);  // U * G < 2^32 (host-checked)
    const int i = (int)((unsigned)u / (unsigned)L);
    return i * L + snap(ph, u - i * L);
  }
  // CTA holding the chunk that starts at tile-local block sl of tile tl: the last jj with
  // bnd(jj) <= tl*L + sl.  snap(u) passes sl once u reaches sl + 7 (or the end of sl's half), so
  // that jj is the last one with floor(U*jj/G) < u_t, i.e. ceil(u_t*G/U) - 1.
  __device__ int owner(int ph, int tl, int sl, int G) const {
    const int L = len(ph), U = (ph == 0 ? T1 : T2) * L;
    int h0, hl;
    half_of(ph, sl, &h0, &hl);
    const unsigned ut = (unsigned)(tl * L + min(sl + kTcChunk / 2, h0 + hl));
    const int jj = (int)((ut * (unsigned)G + (unsigned)U - 1u) / (unsigned)U) - 1;
    return min(max(jj, 0), G - 1);
  }
  // 8-row groups of a tile holding real rows (16, or 8 for a last half tile)
  __device__ int groups(int tile) const {
    const int rows = tile < T1 ? F - 128 * (tile % ns1) : H - 128 * ((tile - T1) % nr2);
    return rows >= 128 ? 16 : rows / 8;
  }
};

// Partial sums CTA `cta` publishes in phase `ph` (at most one tile per phase: the first of its range).
template <int NT>
__device__ __forceinline__ float* tc_partial(float* base, int part_floats, int cta, int ph) {
  return base + (size_t)cta * part_floats + (ph == 0 ? 0 : 2 * NT * 128);
}

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

// Block exponent of a 32-value block with max |v| = m: be = biased fp32 exponent of m, so that
// max |v| < 2^e with e = be - 126.  Blocks below 2^-105 (or all zero) return 0 and are encoded as
// zeros.
__device__ __forceinline__ int block_be(float m) {
  const int be = (int)((__float_as_uint(m) >> 23) & 255u);
  return be >= 22 ? be : 0;
}

// Balanced radix-8 digit planes of one value: X = round(v * 2^(23-e)), |X| <= 2^23, written as
// X = sum_{p<7} d_p 8^p + d_7 8^7 with d_p in [-4, 3] and d_7 in [-4, 4].  Adding
// c = 4 * (8^7 - 1) / 7 makes the seven low digits plain 3-bit fields of X + c (no carries), so all
// planes come out in parallel.  Returns the e2m1 nibble codes (digit d -> value d/2: code |d|,
// bit 3 = sign), plane p in bits 4p..4p+3.
__device__ __forceinline__ uint32_t digit_planes(float v, int be) {
  if (be == 0) return 0u;
  const int X = __float2int_rn(v * __uint_as_float((uint32_t)(276 - be) << 23));  // v * 2^(149-be), exact
  const int Y = X + 1198372;
  uint32_t codes = 0;
#pragma unroll
  for (int p = 0; p < 7; ++p)  // field u = d + 4: code 12-u for u < 4 (negative d), u-4 otherwise
    codes |= ((0x32109ABCu >> (4 * ((Y >> (3 * p)) & 7))) & 15u) << (4 * p);
  const int Q = Y >> 21;  // d_7 in [-4, 4]
  return codes | ((uint32_t)(Q < 0 ? 8 - Q : Q) << 28);
}

// UE8M0 scale of plane p: 2^(3p + e - 22) with bias 127 -> 3p + be - 21 (1..254 for be in 22..254).
__device__ __forceinline__ uint32_t plane_scale(int p, int be) { return be ? (uint32_t)(3 * p + be - 21) : 127u; }

// One half-warp (16 lanes, lane j holds block values v[j] and v[j+16]) writes the
// 8 planes of one block: plane p byte j = code(v[j]) | code(v[j+16]) << 4, to
// dst + p*16 + j; the 8 scale bytes to sdst[p * sstride] (lane 0 of the half).
__device__ __forceinline__ void halfwarp_block_planes(float v0, float v1, uint8_t* dst, uint8_t* sdst, int sstride,
                                                      int hl /*0..15*/, unsigned mask) {
  float m = fmaxf(fabsf(v0), fabsf(v1));
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(mask, m, o, 16));
  const int be = block_be(m);
  const uint32_t c0 = digit_planes(v0, be), c1 = digit_planes(v1, be);
#pragma unroll
  for (int p = 0; p < 8; ++p) {
    const uint32_t b = ((c0 >> (4 * p)) & 15u) | (((c1 >> (4 * p)) & 15u) << 4);
    dst[p * 16 + hl] = (uint8_t)b;
  }
  if (hl == 0)
#pragma unroll
    for (int p = 0; p < 8; ++p) sdst[p * sstride] = (uint8_t)plane_scale(p, be);
}

// Phase-1 B operand: the digit planes of h = (x * r) * norm_w, built by 16 warps (32 half-warps,
// index hw) from the copy of h the prologue left in shared memory, while the first weight chunks
// are in flight.  (Reading x again from L2 here queued behind the weight stream for ~4 us.)
// Token t's planes are rows 8t..8t+7: core matrix (t, block b) at b1 + t*nb_h*128 + b*128; scale
// atom b/4 at sfb1 + (b/4)*sfb1_atom, byte 16*(8t+p) + b%4.
__device__ __forceinline__ void tc_build_b1(const float* h, int H, int T, int nb_h, uint8_t* b1, uint8_t* sfb1,
                                            int sfb1_atom, int hw, int lane) {
  const int hl = lane & 15;
  const unsigned mask = 0xFFFFu << (lane & 16);
  const int nit = T * nb_h;
  for (int it = hw; it < nit; it += 32) {
    const int t = it / nb_h, b = it - t * nb_h;
    const float* hb = h + (int64_t)t * H + 32 * b + hl;
    halfwarp_block_planes(hb[0], hb[16], b1 + (size_t)t * nb_h * 128 + b * 128,
                          sfb1 + (b >> 2) * sfb1_atom + 16 * (8 * t) + (b & 3), 16, hl, mask);
  }
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
  uint8_t* b2 = smem + a.off_b2;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + a.off_bars);
  uint64_t* full_raw = bars;
  uint64_t* empty_raw = full_raw + TcRaw<NT>::kStages;
  uint64_t* full_can = empty_raw + TcRaw<NT>::kStages;
  uint64_t* empty_can = full_can + kTcCanStages;
  uint64_t* full_d = empty_can + kTcCanStages;
  uint64_t* empty_d = full_d + 2;
  uint64_t* mma_done = empty_d + 2;
  uint64_t* b1_ready = mma_done + 1;  // phase-1 activation planes built (16 builder warps)
  uint64_t* b2_full = b1_ready + 1;   // a pair's phase-2 image is in shared memory (loader warp)
  uint64_t* b2_empty = b2_full + kTcB2Bufs;  // the MMAs that read an image buffer are done
  TcShared& S = *reinterpret_cast<TcShared*>(smem + a.off_shared);
  volatile int* abort_flag = &S.abort_flag;

  if (tid == 0) {
    stamp(a.trace, kEvStart);
    for (int s = 0; s < TcRaw<NT>::kStages; ++s) {
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
    mbar_init(b1_ready, kTcRepackWarps + 4);
    for (int s = 0; s < kTcB2Bufs; ++s) {
      mbar_init(&b2_full[s], 1);
      mbar_init(&b2_empty[s], 1);
    }
    fence_mbar_init();
    // TMA boxes and operand tiles assume a 1024-byte aligned dynamic shared-memory base
    S.abort_flag = (smem_addr(smem) & 1023u) != 0;
    if (S.abort_flag) raise_device_error(NS_DEVERR_COPY_WAIT);
    prefetch_tmap(&a.tm_gate16);
    prefetch_tmap(&a.tm_up16);
    prefetch_tmap(&a.tm_down16);
  }
  if (warp == kTcMmaWarp) tmem_alloc(&S.tmem_base, kTcTmemCols);

  // ---- 1. x into shared memory, RMSNorm sum of squares, this CTA's router logit.  The layer's own
  // constants (norm weight, this CTA's router row; one pass covers H <= 4096) are loaded before the
  // wait on the previous kernel of the stream: under programmatic dependent launch that wait is
  // where x and the workspace, which the previous layer wrote, become visible.
  static_assert(128 * 32 <= 8 * kTcThreads, "H <= 4096 (moe_tc_eligible) must fit one pass");
  static_assert(2 * 4096 * 4 <= kTcRawBytes, "T x H fp32 (T <= 2, H <= 4096) must fit one raw stage");
  // T x H fp32 in the last raw stage: read by the prologue and the phase-1 plane builders; the
  // producer overwrites it only after b1_ready
  float* h = reinterpret_cast<float*>(raw + (TcRaw<NT>::kStages - 1) * kTcRawBytes);
  const bool own_expert = c < E;
  // the next kernels' weights into L2 while this layer routes (a hint; static data, so before the wait)
  if (tid == kTcThreads - 1) l2_prefetch_share(p.l2, blockIdx.x, gridDim.x);
  float wv[8], rv[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const int i = tid + u * kTcThreads;
    wv[u] = i < H && p.norm_w ? p.norm_w[i] : 1.0f;
  }
  load_floats<8>(p.router_w, p.router_dtype, [&](int u) -> int64_t {
    const int i = tid + u * kTcThreads;
    return i < H && own_expert ? (int64_t)c * H + i : -1;
  }, rv);
  griddep_wait();
  // counters of this launch (used only after the routing barrier)
  if (c == 0) {
    for (int i = tid; i < a.zero_tiles; i += kTcThreads) a.cnt[i] = 0u;
    for (int i = tid; i < kMaxPairs; i += kTcThreads) a.ready[i] = 0u;
    for (int i = tid; i < kTcMaxRowTiles; i += kTcThreads) a.cnt2[i] = 0u;
  }
  for (int t = 0; t < T; ++t) {
    float ss = 0.f, dot = 0.f;
    float xv[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {  // 8 loads in flight per thread, then the sums in order
      const int i = tid + u * kTcThreads;
      xv[u] = i < H ? p.x[(int64_t)t * H + i] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = tid + u * kTcThreads;
      if (i < H) {
        h[t * H + i] = xv[u];
        ss = fmaf(xv[u], xv[u], ss);
        dot = fmaf(xv[u] * wv[u], rv[u], dot);
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
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = tid + u * kTcThreads;
      if (i < H)
        for (int t = 0; t < T; ++t) h[t * H + i] = __fmul_rn(__fmul_rn(h[t * H + i], S.rscale[t]), wv[u]);
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

  // ---- 2. grid barrier: every CTA's router logit is in the workspace
  if (tid == 0) {
    stamp(a.trace, kEvRouter);
    __threadfence();
    const unsigned long long old = atomicAdd(a.bar, 1ull);
    S.bar_target = (old / (unsigned)G + 1ull) * (unsigned)G;
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
    // every CTA of this layer is past its reads of the previous layer's results: the next kernel in
    // the stream may start its CTAs as SMs free up (they wait for this grid before reading x)
    griddep_launch_dependents();
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
  }
  if (tid == 0) stamp(a.trace, kEvTopk);

  // ---- 4 + 5, in parallel: warp 0 finishes routing (weights, slots, pairs); warp 1 derives this
  // CTA's work.  Lane l = t*k + j holds routed expert (t, j); T*k <= 32 for this kernel.
  if (warp == 0 || warp == 1) {
    const int nall = T * k;
    const bool act = lane < nall;
    const int t = (T == 2 && lane >= k) ? 1 : 0, j = lane - t * k;
    const int e = act ? S.ids[t][j] : 0x7FFFFFFF;
    const bool loc = act && e >= p.expert_lo && e < p.expert_hi;
    int less_local = 0, same_before = 0;
    for (int l2 = 0; l2 < nall; ++l2) {
      const int e2 = __shfl_sync(0xffffffffu, e, l2);
      if (e2 < p.expert_lo || e2 >= p.expert_hi) continue;
      less_local += e2 < e;
      same_before += (e2 == e && l2 < lane);
    }
    const bool first = loc && same_before == 0;
    const unsigned first_mask = __ballot_sync(0xffffffffu, first);
    const int npairs = __popc(__ballot_sync(0xffffffffu, loc)), nslots = __popc(first_mask);
    if (warp == 0) {
      // routing weights: GPT-OSS softmax over the k (neurostream/model/gpt_oss.py:119-120); Qwen3
      // renormalised top-k probabilities (neurostream/moe/router.py:66-68)
      const float v = act ? S.topv[t][j] : 0.f;
      const float mx = __shfl_sync(0xffffffffu, v, t * k);
      float wgt;
      if (p.route_mode == NS_ROUTE_TOPK_SOFTMAX) {
        const float ex = act ? expf(v - mx) : 0.f;
        float sum = 0.f;
        for (int l2 = 0; l2 < nall; ++l2) {  // per-token sum, fixed order
          const float x2 = __shfl_sync(0xffffffffu, ex, l2);
          if (l2 >= t * k && l2 < t * k + k) sum += x2;
        }
        wgt = ex / sum;
      } else {
        float sum = 0.f;
        for (int l2 = 0; l2 < nall; ++l2) {
          const float x2 = __shfl_sync(0xffffffffu, v, l2);
          if (l2 >= t * k && l2 < t * k + k) sum += x2;
        }
        wgt = v / sum;
      }
      if (act) S.w[t][j] = wgt;
      int distinct_less = 0;
      for (int l2 = 0; l2 < nall; ++l2) {
        const int e2 = __shfl_sync(0xffffffffu, e, l2);
        distinct_less += ((first_mask >> l2) & 1u) && e2 < e;
      }
      if (loc) {
        const int pidx = less_local + same_before;
        S.pair_token[pidx] = t;
        S.pair_w[pidx] = wgt;
        S.pair_slot[pidx] = distinct_less;
        if (first) {
          S.slot_expert[distinct_less] = e;
          S.slot_pair0[distinct_less] = less_local;
        }
      }
      if (lane == 0) {
        S.slot_pair0[nslots] = npairs;
        S.nslots = nslots;
        S.npairs = npairs;
      }
      if (c == 0 && act) {
        if (p.ids) p.ids[lane] = e;
        if (p.weights) p.weights[lane] = wgt;
      }
    } else {
      // this CTA's segments: each phase's K blocks split evenly over the CTAs at chunk boundaries
      TcGeom g;
      g.ns1 = (F + 127) / 128;
      g.nr2 = (H + 127) / 128;
      g.T1 = nslots * g.ns1;
      g.T2 = npairs * g.nr2;
      g.nb_h = a.nb_h;
      g.nb_f = a.nb_f;
      g.H = H;
      g.F = F;
      int n[2], lo[2], hi[2];
      for (int ph = 0; ph < 2; ++ph) {
        const int L = g.len(ph);
        lo[ph] = g.bnd(ph, c, G);
        hi[ph] = g.bnd(ph, c + 1, G);
        n[ph] = hi[ph] > lo[ph] ? (hi[ph] - 1) / L - lo[ph] / L + 1 : 0;
      }
      const int ns = n[0] + n[1];
      if (ns > kTcMaxSegs) {
        if (lane == 0) {
          raise_device_error(NS_DEVERR_ROUTE);
          S.abort_flag = 1;
        }
      } else if (lane < ns) {
        const int ph = lane < n[0] ? 0 : 1, li = ph == 0 ? lane : lane - n[0];
        const int L = g.len(ph);
        const int tl = lo[ph] / L + li;  // tile within the phase
        const int s0 = tl * L, e0 = s0 + L;
        TcSeg& sg = S.seg[lane];
        sg.tile = ph == 0 ? tl : g.T1 + tl;
        sg.k0 = max(lo[ph], s0) - s0;
        sg.k1 = min(hi[ph], e0) - s0;
        sg.grp = ph == 0 ? tl / g.ns1 : tl / g.nr2;       // slot (phase 1) or pair (phase 2)
        sg.sub = ph == 0 ? tl - sg.grp * g.ns1 : tl - sg.grp * g.nr2;  // 128-row block within it
      }
      if (lane == 0) {
        S.nseg = ns > kTcMaxSegs ? 0 : ns;
        stamp(a.trace, kEvRoute);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid == 0) stamp(a.trace, kEvLogits);  // every warp knows the routed work

  TcGeom geo;
  geo.ns1 = (F + 127) / 128;
  geo.nr2 = (H + 127) / 128;
  geo.T1 = S.nslots * geo.ns1;
  geo.T2 = S.npairs * geo.nr2;
  geo.nb_h = a.nb_h;
  geo.nb_f = a.nb_f;
  geo.H = H;
  geo.F = F;

  const int nseg = S.nseg;
  const uint32_t tbase = S.tmem_base;

  // Chunks of a segment: [kb, kb + nbc) within one half of the tile (gate or up for phase 1).
  auto chunk_of = [&](int ph, int kb, int k1, int* w, int* nbc, bool* up) {
    int h0, hl;
    geo.half_of(ph, kb, &h0, &hl);
    *w = kb - h0;
    *nbc = min(min(kTcChunk, hl - *w), k1 - kb);
    *up = ph == 0 && h0 > 0;
  };

  // ---- no routed local expert (expert parallel): this rank contributes zeros (+ residual)
  if (S.npairs == 0) {
    const int r0 = (int)((int64_t)H * c / G), r1 = (int)((int64_t)H * (c + 1) / G);
    for (int q = tid; q < T * (r1 - r0); q += kTcThreads) {
      const int t = q / (r1 - r0), r = r0 + (q - t * (r1 - r0));
      p.out[(int64_t)t * H + r] = p.add_residual ? p.x[(int64_t)t * H + r] : 0.f;
    }
  } else if (warp == kTcProducerWarp) {
    // ================================================================= producer (TMA)
    if (lane == 0) {
      const uint64_t policy = l2_evict_first_policy();
      int n = 0;
      for (int sgi = 0; sgi < nseg && !*abort_flag; ++sgi) {
        const TcSeg& sg = S.seg[sgi];
        const int i = sg.tile, ph = i < geo.T1 ? 0 : 1, gv = geo.groups(i);
        const int rb = ph == 0 ? a.rb_h : a.rb_f;
        const int el = S.slot_expert[ph == 0 ? sg.grp : S.pair_slot[sg.grp]] - p.expert_lo;
        const int y0 = ((ph == 0 ? el * F : el * H) + 128 * sg.sub) / 8;
        const int k1 = sg.k1;
        for (int kb = sg.k0; kb < k1 && !*abort_flag; ++n) {
          int w, nbc;
          bool up;
          chunk_of(ph, kb, k1, &w, &nbc, &up);
          const CUtensorMap* tm = ph == 1 ? (gv == 16 ? &a.tm_down16 : &a.tm_down8)
                                          : up ? (gv == 16 ? &a.tm_up16 : &a.tm_up8)
                                               : (gv == 16 ? &a.tm_gate16 : &a.tm_gate8);
          const int st = n % TcRaw<NT>::kStages;
          // the last stage holds h until the phase-1 planes are built
          if (n == TcRaw<NT>::kStages - 1 && !tc_wait(b1_ready, 0, abort_flag)) break;
          if (!tc_wait(&empty_raw[st], ((n / TcRaw<NT>::kStages) & 1) ^ 1, abort_flag)) break;
          mbar_arrive_expect_tx(&full_raw[st], (uint32_t)(8 * gv * kTcBoxW));
          uint8_t* dst = raw + st * kTcRawBytes;
#pragma unroll 1
          for (int j = 0; j < 8; ++j) {
            const int x0 = ((j * rb + 17 * w) & ~15) >> 1;  // u16 elements
            tma_load_2d_hint(dst + j * kTcBoxBytes, tm, x0, y0, &full_raw[st], policy);
          }
          if (n == 0) stamp(a.trace, kEvProducerFirst);
          kb += nbc;
        }
      }
      // let every issued load land before the CTA can exit
      for (int q = max(0, n - TcRaw<NT>::kStages); q < n; ++q)
        mbar_wait_bounded(&full_raw[q % TcRaw<NT>::kStages], (q / TcRaw<NT>::kStages) & 1);
      stamp(a.trace, kEvProducerLast);
    }
  } else if (warp == kTcLoaderWarp) {
    // ---- phase-2 activation images: for each pair this CTA's phase-2 segments use (in order),
    // lane 0 waits until all its phase-1 tiles are counted done (and the MMAs that read the target
    // buffer's previous pair are done); then the warp copies the image from L2 into the next of two
    // buffers with cp.async (plain loads: the epilogues that wrote it need no proxy fence) and hands
    // it to the tensor core (proxy fence, then one arrival)
    const int n16 = (a.nb_f * 128 + (a.nb_f + 3) / 4 * 128) / 16;
    int k2 = 0, prev = -1;
    for (int sgi = 0; sgi < nseg; ++sgi) {
      const TcSeg& sg = S.seg[sgi];
      if (sg.tile < geo.T1 || sg.grp == prev) continue;
      const int pp = sg.grp, buf = k2 % kTcB2Bufs;
      int ok = 1;
      if (lane == 0) {
        if (k2 >= kTcB2Bufs && !tc_wait(&b2_empty[buf], ((k2 / kTcB2Bufs) - 1) & 1, abort_flag)) ok = 0;
        const unsigned* rdy = a.ready + S.pair_slot[pp];
        const uint64_t t0 = globaltimer_ns();
        while (ok && ld_acquire_u32(rdy) < (unsigned)geo.ns1) {
          if (*abort_flag || globaltimer_ns() - t0 > kWaitLimitNs) {
            if (!*abort_flag) raise_device_error(NS_DEVERR_GRID_WAIT);
            *abort_flag = 1;
            ok = 0;
          }
          __nanosleep(32);
        }
        if (ok && k2 == 0) stamp(a.trace, kEvBarrier2);
      }
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;  // the whole warp leaves together
      // lane 0's acquire, then this warp barrier: the other CTAs' image stores are visible to every lane
      __syncwarp();
      const uint4* src = reinterpret_cast<const uint4*>(a.actimg + (size_t)pp * a.img_bytes);
      uint4* dst = reinterpret_cast<uint4*>(b2 + buf * a.b2_stride);
      for (int i = lane; i < n16; i += 32) cp_async16(dst + i, src + i);
      cp_async_commit();
      cp_async_wait<0>();
      fence_proxy_async_smem();  // generic-proxy writes to shared memory -> read by the MMAs
      __syncwarp();
      if (lane == 0) mbar_arrive(&b2_full[buf]);
      ++k2;
      prev = pp;
    }
  } else if (warp == kTcMmaWarp) {
    // ================================================================= MMA issuer
    if (lane == 0) {
      int n = 0;
      bool have_b1 = false;
      int k2 = -1, prev2 = -1;  // phase-2 pairs met so far (image buffer k2 % kTcB2Bufs), current pair
      uint32_t sfb2_have = 0u;  // scale atoms of the current pair already in TMEM (nb_f <= 128: <= 32)
      for (int sgi = 0; sgi < nseg && !*abort_flag; ++sgi) {
        const TcSeg& sg = S.seg[sgi];
        const int i = sg.tile, ph = i < geo.T1 ? 0 : 1;
        const int db = sgi & 1;
        if (ph == 0 && !have_b1) {
          if (!tc_wait(b1_ready, 0, abort_flag)) break;
          tc_fence_after();
          for (int at = 0; at < (a.nb_h + 3) / 4; ++at)  // phase-1 activation scales, once per launch
            tc_cp_sf(tbase + kTcTmemSfb1 + 4 * at, umma_desc(smem_addr(sfb1 + at * a.sfb1_atom), 128, 128));
          have_b1 = true;
        }
        if (ph == 1 && sg.grp != prev2) {  // a new pair: its image must be in shared memory
          ++k2;
          prev2 = sg.grp;
          sfb2_have = 0u;
          if (!tc_wait(&b2_full[k2 % kTcB2Bufs], (k2 / kTcB2Bufs) & 1, abort_flag)) break;
          tc_fence_after();
          if (k2 == 0) stamp(a.trace, kEvImages);
        }
        if (!tc_wait(&empty_d[db], ((sgi >> 1) & 1) ^ 1, abort_flag)) break;
        const uint32_t tmem_d = tbase + kTcDCols * db;
        const int N = ph == 0 ? 8 * NT : 8;
        bool fresh_gate = true, fresh_up = true;  // accumulators not yet written in this segment
        const int k1 = sg.k1;
        bool ok = true;
        for (int kb = sg.k0; kb < k1; ++n) {
          int w, nbc;
          bool up;
          chunk_of(ph, kb, k1, &w, &nbc, &up);
          const int st = n % kTcCanStages;
          if (!tc_wait(&full_can[st], (n / kTcCanStages) & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sfa_col = tbase + kTcTmemSfa + 16 * st;  // written by the repack warps
          const uint32_t a_col = tbase + kTcTmemA + kTcTmemAStage * st;
          const uint32_t dcol = tmem_d + (up ? 16 : 0);
          // B: the resident activation planes (phase 1: the token's, phase 2: the pair's image).
          // Descriptors advance by 256 bytes (2 blocks of 128 B) per MMA: +16 in the address field.
          const uint64_t db0 =
              ph == 0 ? umma_desc(smem_addr(b1) + (uint32_t)w * 128u, 128, a.nb_h * 128)
                      : umma_desc(smem_addr(b2 + (k2 % kTcB2Bufs) * a.b2_stride) + (uint32_t)w * 128u, 128, a.nb_f * 128);
          const uint32_t sfb_base = tbase + (ph == 0 ? kTcTmemSfb1 : kTcTmemSfb2);
          if (ph == 1) {
            // the pair's activation scales this chunk needs, copied into TMEM on first use (after
            // the previous pair's MMAs: tcgen05 operations of one thread run in issue order)
            const uint8_t* sc = b2 + (k2 % kTcB2Bufs) * a.b2_stride + a.nb_f * 128;
            for (int at = w >> 2; at <= (w + nbc - 1) >> 2; ++at)
              if (!((sfb2_have >> at) & 1u)) {
                tc_cp_sf(sfb_base + 4 * at, umma_desc(smem_addr(sc + at * 128), 128, 128));
                sfb2_have |= 1u << at;
              }
          }
          const uint32_t idesc0 = idesc_mxf4(128, N, 0, 0);
          bool acc = up ? !fresh_up : !fresh_gate;
#pragma unroll
          for (int s = 0; s < kTcChunk / 2; ++s) {
            if (s < nbc / 2) {
              // weight scales: atom s/2 of the chunk; activation scales: the resident atom of block
              // w + 2s (w even)
              const uint32_t sfa_id = 2u * (s & 1);
              const int blk = w + 2 * s;
              const uint32_t sfb_id = (uint32_t)(blk & 3);
              const uint32_t tsfa = (sfa_col + 4 * (s >> 1)) | (sfa_id << 30);
              const uint32_t tsfb = (sfb_base + 4 * (blk >> 2)) | (sfb_id << 30);
              mma_mxf4_ts(dcol, a_col + 8 * s, db0 + (uint64_t)(16 * s), idesc0 | (sfb_id << 4) | (sfa_id << 29),
                          tsfa, tsfb, acc ? 1u : 0u);
              acc = true;
            }
          }
          if (up) fresh_up = false; else fresh_gate = false;
          tc_commit(&empty_can[st]);
          kb += nbc;
        }
        if (!ok) break;
        tc_commit(&full_d[db]);
        if (ph == 0 && (sgi + 1 == nseg || S.seg[sgi + 1].tile >= geo.T1)) stamp(a.trace, kEvPhase1End);
        // the pair's last segment here: its image buffer may be refilled once these MMAs are done
        if (ph == 1 && (sgi + 1 == nseg || S.seg[sgi + 1].grp != prev2)) tc_commit(&b2_empty[k2 % kTcB2Bufs]);
      }
      stamp(a.trace, kEvPhase2Images);
      tc_commit(mma_done);
      mbar_wait_bounded(mma_done, 0);
    }
  } else if (tc_repack_index(warp) >= 0) {
    // ================================================================= repack warps
    // Quadrant q's three warps own M-rows 32q .. 32q+31 (this lane: M-row m, tile row (G, j)) and
    // split a chunk's 14 blocks on scale-atom boundaries: {0-3, 12-13}, {4-7}, {8-11}.  Each
    // block: 5 word loads of the staged row, the 16 payload bytes to 4 TMEM columns of row m; the
    // E8M0 bytes of a 4-block atom form one TMEM word of row m (lane m, column 4*atom + m/32).
    const int rw = tc_repack_index(warp);  // 0..11
    tc_build_b1(h, H, T, a.nb_h, b1, sfb1, a.sfb1_atom, 2 * rw + (lane >> 4), lane);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(b1_ready);
    const int q = rw / 3, wi = rw - 3 * q;
    const int m = 32 * q + lane;
    const int Gr = 8 * (q >> 1) + (lane & 7), j = 2 * (lane >> 3) + (q & 1);
    const uint32_t taddr_lane = (uint32_t)(32 * q) << 16;
    (void)m;
    int n = 0;
    for (int sgi = 0; sgi < nseg && !*abort_flag; ++sgi) {
      const TcSeg& sg = S.seg[sgi];
      const int i = sg.tile, ph = i < geo.T1 ? 0 : 1, gv = geo.groups(i);
      const int rb = ph == 0 ? a.rb_h : a.rb_f;
      const bool row_ok = Gr < gv;
      const int k1 = sg.k1;
      for (int kb = sg.k0; kb < k1 && !*abort_flag; ++n) {
        int w, nbc;
        bool up;
        chunk_of(ph, kb, k1, &w, &nbc, &up);
        const int st = n % TcRaw<NT>::kStages, cst = n % kTcCanStages;
        if (!tc_wait(&full_raw[st], (n / TcRaw<NT>::kStages) & 1, abort_flag)) break;
        if (n == 0 && rw == 0 && lane == 0) stamp(a.trace, kEvFirstTile);
        const uint8_t* rs = raw + st * kTcRawBytes + j * kTcBoxBytes + Gr * kTcBoxW + ((j * rb + 17 * w) & 15);
        // this warp's blocks: u -> b = u (u < 4) or u + 8 for warp 0, 4*wi + u otherwise
        constexpr int kU = 6;
        uint32_t wv[kU][5];
#pragma unroll
        for (int u = 0; u < kU; ++u) {  // all loads first
          const int b = wi == 0 ? (u < 4 ? u : u + 8) : 4 * wi + u;
          const bool ok = row_ok && (wi == 0 || u < 4) && b < nbc;
          const uintptr_t src = reinterpret_cast<uintptr_t>(rs + 17 * b);
          const uint32_t* wp = reinterpret_cast<const uint32_t*>(src & ~uintptr_t(3));
#pragma unroll
          for (int k = 0; k < 5; ++k) wv[u][k] = ok ? wp[k] : 0u;
        }
        uint32_t pay[4 * kU], sw[2] = {0u, 0u};
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int b = wi == 0 ? (u < 4 ? u : u + 8) : 4 * wi + u;
          const uint32_t a0 = (uint32_t)(reinterpret_cast<uintptr_t>(rs + 17 * b) & 3);  // scale byte's offset
          const uint32_t sh = 8 * ((a0 + 1) & 3);
          const bool whole = a0 == 3;  // payload is word-aligned: words 1..4
#pragma unroll
          for (int k = 0; k < 4; ++k)
            pay[4 * u + k] = whole ? wv[u][k + 1] : __funnelshift_r(wv[u][k], wv[u][k + 1], sh);
          sw[u >> 2] |= ((wv[u][0] >> (8 * a0)) & 0xFFu) << (8 * (u & 3));
        }
        __syncwarp();  // every lane has consumed its staged words: the raw stage can be refilled
        if (lane == 0) mbar_arrive(&empty_raw[st]);
        // the operand stage (its A and SFA columns in TMEM) must have been consumed by its earlier MMAs
        if (!tc_wait(&empty_can[cst], ((n / kTcCanStages) & 1) ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t acol = tbase + kTcTmemA + kTcTmemAStage * cst + taddr_lane;
        const uint32_t scol = tbase + kTcTmemSfa + 16 * cst + q + taddr_lane;  // column 4*atom + m/32
        {
          uint32_t v16[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) v16[k] = pay[k];
          tmem_st_x16(acol + 16 * wi, v16);                // blocks 4wi .. 4wi+3
          tmem_st_x1(scol + 4 * wi, sw[0]);                 // their scale atom
          if (wi == 0) {
            uint32_t v8[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) v8[k] = pay[16 + k];
            tmem_st_x8(acol + 48, v8);                      // blocks 12, 13
            tmem_st_x1(scol + 12, sw[1]);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&full_can[cst]);
        }
        kb += nbc;
      }
    }
  } else if (tc_epi_quadrant(warp) >= 0) {
    // ================================================================= epilogue warps
    const int q = tc_epi_quadrant(warp);  // TMEM lane quadrant (= warp % 4)
    const int mrow = 32 * q + lane;       // M-row (TMEM lane) of this thread
    const int row = tc_row_of(mrow);      // the tile row it holds
    const int et = mrow;                  // 0..127
    float* xchg = reinterpret_cast<float*>(smem + a.off_xchg);
    tc_build_b1(h, H, T, a.nb_h, b1, sfb1, a.sfb1_atom, 2 * (kTcRepackWarps + q) + (lane >> 4), lane);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(b1_ready);
    for (int sgi = 0; sgi < nseg; ++sgi) {
      const TcSeg& sg = S.seg[sgi];
      const int i = sg.tile, ph = i < geo.T1 ? 0 : 1;
      const int db = sgi & 1;
      // this row's biases, fetched while the tile's MMAs run
      float bias0 = 0.f, bias1 = 0.f;
      if (ph == 0) {
        const int el = S.slot_expert[i / geo.ns1] - p.expert_lo, n = 128 * (i % geo.ns1) + row;
        if (n < F) {
          if (p.gate_b) bias0 = p.gate_b[(int64_t)el * F + n];
          if (p.up_b) bias1 = p.up_b[(int64_t)el * F + n];
        }
      } else {
        const int qq = i - geo.T1, r = 128 * (qq % geo.nr2) + row;
        const int el = S.slot_expert[S.pair_slot[qq / geo.nr2]] - p.expert_lo;
        if (r < H && p.down_b) bias0 = p.down_b[(int64_t)el * H + r];
      }
      // ---- split tile, finishing side: find the other sharers and sum their partials (published at
      // the start of their ranges) while this CTA's own MMAs for the tile are still running
      const int L = geo.len(ph);
      const bool split = !(sg.k0 == 0 && sg.k1 == L), finisher = sg.k0 == 0;
      float pre[2 * NT];
#pragma unroll
      for (int v = 0; v < 2 * NT; ++v) pre[v] = 0.f;
      if (split && finisher) {
        if (q == 0) {
          const int nq = geo.nchunks(ph), tl = ph == 0 ? i : i - geo.T1;
          const int cc = lane < nq ? geo.owner(ph, tl, geo.chunk_start(ph, lane), G) : -1;
          const int prev = __shfl_up_sync(0xffffffffu, cc, 1);
          const bool nw = lane > 0 && lane < nq && cc != prev;  // owners ascend; chunk 0 is this CTA's
          const unsigned m = __ballot_sync(0xffffffffu, nw);
          if (nw) S.sh_cta[__popc(m & ((1u << lane) - 1u))] = (short)cc;
          if (lane == 0) S.nsh = __popc(m);
        }
        named_sync(1, 128);
        const int nsh = S.nsh;
        if (et == 0) {  // each sharer adds 1 after publishing
          const uint64_t t0 = globaltimer_ns();
          while (ld_acquire_u32(a.cnt + i) < (unsigned)nsh) {
            if (*abort_flag) break;
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
              raise_device_error(NS_DEVERR_GRID_WAIT);
              *abort_flag = 1;
              break;
            }
            __nanosleep(32);
          }
        }
        named_sync(1, 128);
        const int nv0 = ph == 0 ? 2 * NT : 1;
        for (int g0 = 0; g0 < nsh; g0 += 4) {  // four sharers' loads in flight, then summed in order
          float pv[4][2 * NT];
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const bool ok = g0 + g < nsh;
            const float* pg = tc_partial<NT>(a.partial, a.part_floats, ok ? S.sh_cta[g0 + g] : c, ph);
#pragma unroll
            for (int v = 0; v < 2 * NT; ++v) pv[g][v] = ok && v < nv0 ? __ldcg(pg + v * 128 + mrow) : 0.f;
          }
#pragma unroll
          for (int g = 0; g < 4; ++g)
#pragma unroll
            for (int v = 0; v < 2 * NT; ++v)
              if (g0 + g < nsh) pre[v] += pv[g][v];
        }
      }
      if (!tc_wait(&full_d[db], (sgi >> 1) & 1, abort_flag)) break;
      tc_fence_after();
      // vals: phase 1 gate[t] at t, up[t] at NT + t; phase 2 the down row at 0
      float vals[2 * NT];
      const uint32_t ta = tbase + kTcDCols * db + ((uint32_t)(32 * q) << 16);
      if (ph == 0) {
        uint32_t v[16], u[16];
        tmem_ld_x16(ta, v);
        tmem_ld_x16(ta + 16, u);
        tmem_wait_ld();
        const bool has_gate = sg.k0 < geo.nb_h, has_up = sg.k1 > geo.nb_h;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          float sg_ = 0.f, su = 0.f;
#pragma unroll
          for (int pl = 0; pl < 8; ++pl) {
            sg_ += __uint_as_float(v[8 * t + pl]);
            su += __uint_as_float(u[8 * t + pl]);
          }
          vals[t] = has_gate ? sg_ : 0.f;
          vals[NT + t] = has_up ? su : 0.f;
        }
      } else {
        uint32_t v[8];
        tmem_ld_x8(ta, v);
        tmem_wait_ld();
        float s = 0.f;
#pragma unroll
        for (int pl = 0; pl < 8; ++pl) s += __uint_as_float(v[pl]);
#pragma unroll
        for (int t = 0; t < 2 * NT; ++t) vals[t] = t == 0 ? s : 0.f;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_d[db]);
      const int nv = ph == 0 ? 2 * NT : 1;

      if (split && !finisher) {
        // ---- split tile, publishing side: this CTA's partial sums, then one count on the tile
        float* part = tc_partial<NT>(a.partial, a.part_floats, c, ph);
#pragma unroll
        for (int v = 0; v < 2 * NT; ++v)
          if (v < nv) __stcg(part + v * 128 + mrow, vals[v]);
        named_sync(1, 128);
        if (et == 0) red_add_release(a.cnt + i, 1u);
        continue;
      }
      if (split) {  // finishing side: own sum first, then the sharers' in CTA order
#pragma unroll
        for (int v = 0; v < 2 * NT; ++v) vals[v] += pre[v];
      }

      if (ph == 0) {
        // ---- phase-1 tile: neuron 128*sl + row; activations regrouped through shared memory so
        // that warp q writes the planes of neurons 32q .. 32q+31 (block 4*sl + q)
        const int s = i / geo.ns1, sl = i % geo.ns1;
        const int n = 128 * sl + row;
        const int blk = 4 * sl + q;
        for (int pp = S.slot_pair0[s]; pp < S.slot_pair0[s + 1]; ++pp) {
          const int t = S.pair_token[pp];
          float gv_ = 0.f, uv_ = 0.f;
#pragma unroll
          for (int tt = 0; tt < NT; ++tt)
            if (tt == t) {
              gv_ = vals[tt];
              uv_ = vals[NT + tt];
            }
          xchg[row] = n < F ? activate(p.act_mode, gv_ + bias0, uv_ + bias1, p.alpha, p.limit) : 0.f;
          named_sync(1, 128);
          if (32 * blk < F) {  // whole warps: F is a multiple of 64
            const float av = xchg[32 * q + lane];
            float m = fabsf(av);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            const int be = block_be(m);
            const uint32_t cd = digit_planes(av, be);
            const uint32_t hi = __shfl_down_sync(0xffffffffu, cd, 16);
            uint8_t* img = a.actimg + (size_t)pp * a.img_bytes;
            if (lane < 16) {
#pragma unroll
              for (int pl = 0; pl < 8; ++pl) {
                const uint32_t bv = ((cd >> (4 * pl)) & 15u) | (((hi >> (4 * pl)) & 15u) << 4);
                img[(size_t)blk * 128 + pl * 16 + lane] = (uint8_t)bv;
              }
            } else if (lane < 24) {  // scale atom blk/4: row pl, byte blk%4 (tcgen05.cp source layout)
              const int pl = lane - 16;
              img[(size_t)a.nb_f * 128 + (size_t)(blk >> 2) * 128 + 16 * pl + (blk & 3)] = (uint8_t)plane_scale(pl, be);
            }
          }
          named_sync(1, 128);  // xchg is reused by the next pair
        }
        named_sync(1, 128);
        if (et == 0) red_add_release(a.ready + s, 1u);
      } else {
        // ---- phase-2 tile: down rows of one pair; the last pair of a row block combines it
        const int qq = i - geo.T1, pp = qq / geo.nr2, rt = qq % geo.nr2;
        const int r = 128 * rt + row;
        if (r < H) __stcg(a.yp + (size_t)pp * H + r, vals[0] + bias0);
        named_sync(1, 128);
        if (et == 0) {
          const unsigned old = atom_add_acq_rel(a.cnt2 + rt, 1u);
          S.fin = old == (unsigned)(S.npairs - 1);
        }
        named_sync(1, 128);
        if (S.fin) {
          if (r < H)
            for (int t = 0; t < T; ++t) {
              const float xr = p.add_residual ? p.x[(int64_t)t * H + r] : 0.f;
              const int np = S.npairs;
              float o = 0.f;
              for (int q0 = 0; q0 < np; q0 += 8) {  // eight pairs' loads in flight, then summed in order
                float yv[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                  const int q2 = q0 + u;
                  yv[u] = q2 < np && S.pair_token[q2] == t ? __ldcg(a.yp + (size_t)q2 * H + r) : 0.f;
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                  const int q2 = q0 + u;
                  if (q2 < np && S.pair_token[q2] == t) o = __fadd_rn(o, __fmul_rn(S.pair_w[q2], yv[u]));
                }
              }
              p.out[(int64_t)t * H + r] = p.add_residual ? __fadd_rn(xr, o) : o;
            }
        }
      }
    }
    if (et == 0) stamp(a.trace, kEvTilesEnd);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kTcMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tbase, kTcTmemCols);
  }
  if (tid == 0) stamp(a.trace, kEvEnd);
}

// ----------------------------------------------------------------------------- host side

struct TcPlan {
  size_t ws_total;
  size_t off_logits, off_partial, off_img, off_yp;
  int img_bytes, max_tiles, grid, part_floats;
};

// Layers the tensor-core kernel takes: MXFP4 experts, T <= 2, H and F multiples of 64, tiles of
// a phase split over at most kTcMaxSplit CTAs, 16-byte aligned expert tensors (moe_tc_aligned).
static size_t moe_tc_smem(const ns_moe_layer_t* p, MoeTcArgs* a);

static bool moe_tc_eligible(const ns_moe_layer_t* p) {
  if (p->ggml_type != NS_GGML_MXFP4 || p->T > 2) return false;
  if (p->H % 64 || p->F % 64) return false;
  // resident activation scales: 4 TMEM columns per 4 blocks, 128 columns for each phase
  if (p->H / 32 > 128 || p->F / 32 > 128) return false;
  // a tile is shared by at most one CTA per chunk
  const int ch1 = 2 * ((p->H / 32 + kTcChunk - 1) / kTcChunk), ch2 = (p->F / 32 + kTcChunk - 1) / kTcChunk;
  if (ch1 > kTcMaxSplit || ch2 > kTcMaxSplit) return false;
  if (p->T * p->k > kMaxPairs || p->T * p->k > 32) return false;
  const int pairs = p->T * p->k;
  const int64_t tiles = (int64_t)pairs * ((p->F + 127) / 128) + (int64_t)pairs * ((p->H + 127) / 128);
  if (tiles > kTcMaxTiles || (p->H + 127) / 128 > kTcMaxRowTiles) return false;
  // per-phase K blocks times the grid must fit 32 bits (the kernel's range arithmetic)
  const int64_t u1 = (int64_t)pairs * ((p->F + 127) / 128) * 2 * (p->H / 32);
  const int64_t u2 = (int64_t)pairs * ((p->H + 127) / 128) * (p->F / 32);
  if (std::max(u1, u2) * kTcGridMax >= ((int64_t)1 << 32)) return false;
  MoeTcArgs layout;
  return moe_tc_smem(p, &layout) <= (size_t)kTcSmemBudget;
}

static bool moe_tc_aligned(const ns_moe_layer_t* p) {
  auto al = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  return al(p->gate_w) && al(p->up_w) && al(p->down_w);
}

static void moe_tc_plan(const ns_moe_layer_t* p, int grid, TcPlan* t) {
  const int pairs = p->T * p->k;
  const int nb_f = p->F / 32;
  t->grid = grid;
  t->part_floats = (2 * p->T + 1) * 128;
  t->img_bytes = (int)align_up((size_t)nb_f * 128 + (size_t)((nb_f + 3) / 4) * 128, 256);
  t->max_tiles = pairs * ((p->F + 127) / 128) + pairs * ((p->H + 127) / 128);
  size_t off = kTcWsHeader;
  t->off_logits = off;
  off += align_up((size_t)p->T * p->n_expert * 4, 256);
  t->off_partial = off;
  off += align_up((size_t)grid * t->part_floats * 4, 256);
  t->off_img = off;
  off += (size_t)pairs * t->img_bytes;
  t->off_yp = off;
  off += align_up((size_t)pairs * p->H * 4, 256);
  t->ws_total = off;
}

static size_t moe_tc_smem(const ns_moe_layer_t* p, MoeTcArgs* a) {
  const int nb_h = p->H / 32;
  a->off_raw = 0;
  const int raw_stages = p->T == 1 ? TcRaw<1>::kStages : TcRaw<2>::kStages;
  size_t off = std::max((size_t)raw_stages * kTcRawBytes, align_up((size_t)p->T * p->H * 4, 1024));
  off = align_up(off, 1024);
  a->off_b1 = (int)off;
  off += (size_t)p->T * nb_h * 128;
  off = align_up(off, 128);
  a->off_sfb1 = (int)off;
  a->sfb1_atom = 128 * p->T;
  off += (size_t)((nb_h + 3) / 4) * a->sfb1_atom + 512;
  off = align_up(off, 128);
  // phase-2 images: planes, then scale atoms (+512: a scale copy reads 32 rows from its atom on)
  const int nb_f = p->F / 32;
  a->off_b2 = (int)off;
  a->b2_stride = (int)align_up((size_t)nb_f * 128 + (size_t)((nb_f + 3) / 4) * 128 + 512, 128);
  off += (size_t)kTcB2Bufs * a->b2_stride;
  a->off_xchg = (int)off;
  off += 128 * 4;
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

// Tensor map over `rows` GGUF rows of `rb` bytes viewed as (rows/8) groups of 8*rb bytes (16-bit
// elements); the box is 272 bytes of `box_groups` consecutive groups.
static int make_row_group_map(CUtensorMap* m, const uint8_t* base, int64_t rows, int rb, int box_groups) {
  EncodeTiledFn fn;
  int st = get_encode_fn(&fn);
  if (st) return st;
  const cuuint64_t dims[2] = {(cuuint64_t)4 * rb, (cuuint64_t)(rows / 8)};  // u16 elements (rb is even)
  const cuuint64_t strides[1] = {(cuuint64_t)8 * rb};
  const cuuint32_t box[2] = {(cuuint32_t)(kTcBoxW / 2), (cuuint32_t)box_groups};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint8_t*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NS_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return NS_OK;
}

static bool g_tc_pdl = true;  // programmatic dependent launch accepted so far

// The launch is a plain one: with one CTA per SM and a grid of at most the SM count every CTA is
// resident once the stream's previous kernel has left its SMs, and under programmatic dependent
// launch each CTA starts (barrier set-up, TMEM, its router row and the norm weight in flight) as
// soon as its SM frees up instead of all together; the grid-wide waits are bounded, so a grid that
// could not become resident (other work holding SMs for over a second) ends with a device error
// bit rather than hanging.  1 builds a cooperative launch (every CTA resident before any starts).
#ifndef NS_MOE_TC_COOPERATIVE
#define NS_MOE_TC_COOPERATIVE 0
#endif

template <int NT>
static int launch_moe_tc(const MoeTcArgs& a, int grid, size_t smem, cudaStream_t stream) {
  auto kern = moe_tc_kernel<NT>;
  // the kernel's whole budget, not this launch's size (see dense.cu: graphs replay against the attribute)
  NS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)std::max(smem, (size_t)kTcSmemBudget)));
  int per_sm = 0;
  NS_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kTcThreads, smem));
  if (per_sm < 1) return fail(NS_ERR_UNSUPPORTED, "ns_moe_decode_layer: tensor-core kernel does not fit on an SM");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  // Programmatic dependent launch: this grid's CTAs may start while the previous kernel of the
  // stream finishes; the kernel waits for it (griddepcontrol.wait) before reading anything that
  // kernel may have written other than the layer's weights.
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = NS_MOE_TC_COOPERATIVE;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_tc_pdl ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
  if (e != cudaSuccess && g_tc_pdl) {  // runtime without programmatic launch for cooperative grids
    (void)cudaGetLastError();
    g_tc_pdl = false;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, a);
  }
  NS_CUDA_TRY(e);
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
  const int64_t rows_gu = (int64_t)n_local * p->F, rows_d = (int64_t)n_local * p->H;
  int st = make_row_group_map(&a.tm_gate16, p->gate_w, rows_gu, a.rb_h, 16);
  if (!st) st = make_row_group_map(&a.tm_gate8, p->gate_w, rows_gu, a.rb_h, 8);
  if (!st) st = make_row_group_map(&a.tm_up16, p->up_w, rows_gu, a.rb_h, 16);
  if (!st) st = make_row_group_map(&a.tm_up8, p->up_w, rows_gu, a.rb_h, 8);
  if (!st) st = make_row_group_map(&a.tm_down16, p->down_w, rows_d, a.rb_f, 16);
  if (!st) st = make_row_group_map(&a.tm_down8, p->down_w, rows_d, a.rb_f, 8);
  if (st) return st;
  a.bar = reinterpret_cast<unsigned long long*>(ws);
  a.cnt = reinterpret_cast<unsigned*>(ws + kTcOffCnt);
  a.ready = reinterpret_cast<unsigned*>(ws + kTcOffReady);
  a.cnt2 = reinterpret_cast<unsigned*>(ws + kTcOffCnt2);
  a.logits = reinterpret_cast<float*>(ws + tp.off_logits);
  a.partial = reinterpret_cast<float*>(ws + tp.off_partial);
  a.part_floats = tp.part_floats;
  a.actimg = ws + tp.off_img;
  a.yp = reinterpret_cast<float*>(ws + tp.off_yp);
  a.img_bytes = tp.img_bytes;
  a.zero_tiles = tp.max_tiles;
  a.trace = g_trace_buf[trace_slot()];
  const size_t smem = moe_tc_smem(p, &a);
  if (smem > (size_t)kTcSmemBudget)
    return fail(NS_ERR_UNSUPPORTED, "ns_moe_decode_layer: tensor-core layout needs %zu bytes of shared memory", smem);
  if (tp.grid > kTcGridMax) return fail(NS_ERR_UNSUPPORTED, "ns_moe_decode_layer: more than %d SMs", kTcGridMax);
  return p->T == 1 ? launch_moe_tc<1>(a, tp.grid, smem, s) : launch_moe_tc<2>(a, tp.grid, smem, s);
}

}  // namespace ns
