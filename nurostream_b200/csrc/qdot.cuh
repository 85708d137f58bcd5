// Quantized dot products straight from GGUF bytes staged in shared memory.
//
// Every supported format is read as "groups": group g of a row covers the 32
// consecutive elements x[32g .. 32g+31] and decodes from a fixed set of bytes:
//   MXFP4  block g (17 B): E8M0 exponent + 16 payload bytes; byte j holds
//          element j (low nibble) and j+16 (high nibble).
//   Q8_0   block g (34 B): fp16 d + 32 int8.
//   Q4_K   superblock g/8 (144 B), sub-block s = g%8: 32 bytes of qs at
//          16 + 32*(s/2), nibble s%2; 6-bit scale/min from the 12 scale bytes.
//   Q5_K   superblock g/8 (176 B), sub-block s = g%8: as Q4_K with qs at 48 + 32*(s/2) and the
//          fifth bit of element l in bit s of qh byte 16 + l.
//   Q4_0   block g (18 B): fp16 d + 16 bytes; byte j holds element j (low nibble) and
//          j+16 (high nibble), both stored +8.
//   Q6_K   superblock g/8 (210 B), half h = (g/4)%2, lane i = g%4: ql bytes at
//          64h + 32*(i%2) (nibble i/2), qh bytes at 128 + 32h (bits 2i..2i+1),
//          int8 scales at 192 + 8h + 2i (+1 for the second 16 elements), fp16 d at 208.
// These mappings restate the reference decoders (neurostream/compute/quant.py:24-140)
// group by group.  A group is processed as four 8-element sub-chunks so that
// the x values of a sub-chunk are loaded once and reused for R rows.
//
// Arithmetic: products and sums in fp32.  Per group the partial sum
// sum(x * q) is formed first and scaled once (the block scale factors out of
// the group's elements), which is the reference's math in a different
// rounding order.
#pragma once

#include "common.cuh"

namespace ns {

// e2m1 pairs -> fp16x2: 4 bytes of a word, each byte's low nibble to the low half.
__device__ __forceinline__ void e2m1x4_to_f16x2(uint32_t w, uint32_t (&h)[4]) {
  asm("{\n .reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %4;\n"
      " cvt.rn.f16x2.e2m1x2 %0, b0;\n cvt.rn.f16x2.e2m1x2 %1, b1;\n"
      " cvt.rn.f16x2.e2m1x2 %2, b2;\n cvt.rn.f16x2.e2m1x2 %3, b3;\n}"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "r"(w));
}

__device__ __forceinline__ float2 f16x2_to_float2(uint32_t h) {
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}

// Byte i of w (0..255) as an exact float minus `bias`, via the 2^23 trick:
// the word 0x4B0000bb is the float 2^23 + bb.
__device__ __forceinline__ float byte_as_float(uint32_t w, int i, float bias_plus_2p23) {
  return __int_as_float(__byte_perm(w, 0x4B00u, 0x5440u + (unsigned)i)) - bias_plus_2p23;
}

constexpr float k2p23 = 8388608.0f;

// ----------------------------------------------------------------------------- int8 activation planes

// Q8_0 and Q4_K dot products on dp4a: the activations of a 32-element group as three int8 digit
// planes, the balanced radix-256 digits of X = rint(x * 2^(22-e)) with max|x| < 2^e (|X| <= 2^22,
// so every digit fits int8; an exact 22-bit fixed point of the group).  A group's planes take
// kXQG bytes (3 x 32, padded so that lanes reading consecutive groups hit different banks).
constexpr int kXQG = 112;

// v: the group's 32 values.  Writes the planes to grp (16-byte aligned) and returns the group's
// scale 2^(e-22) (0 for groups below 2^-104 or non-finite, which are taken as zeros) and its sum.
__device__ __forceinline__ void group_planes_i8(const float (&v)[32], uint8_t* grp, float* scale, float* sum) {
  float m = 0.f, sm = 0.f;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    m = fmaxf(m, fabsf(v[j]));
    sm += v[j];
  }
  const int be = (int)((__float_as_uint(m) >> 23) & 255u);  // max|x| < 2^e, e = be - 126
  const bool live = be >= 22 && be < 255;
  const float to_fixed = __uint_as_float((uint32_t)(275 - be) << 23);  // 2^(22-e)
  uint32_t pl[3][8] = {};
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int X = live ? __float2int_rn(v[j] * to_fixed) : 0;
    const int d0 = ((X + 128) & 255) - 128;
    const int X1 = (X - d0) >> 8;
    const int d1 = ((X1 + 128) & 255) - 128;
    const int d2 = (X1 - d1) >> 8;
    pl[0][j >> 2] |= (uint32_t)(d0 & 255) << (8 * (j & 3));
    pl[1][j >> 2] |= (uint32_t)(d1 & 255) << (8 * (j & 3));
    pl[2][j >> 2] |= (uint32_t)(d2 & 255) << (8 * (j & 3));
  }
  uint4* out = reinterpret_cast<uint4*>(grp);
#pragma unroll
  for (int p = 0; p < 3; ++p) {
    out[2 * p] = make_uint4(pl[p][0], pl[p][1], pl[p][2], pl[p][3]);
    out[2 * p + 1] = make_uint4(pl[p][4], pl[p][5], pl[p][6], pl[p][7]);
  }
  *scale = live ? __uint_as_float((uint32_t)(be - 21) << 23) : 0.f;  // 2^(e-22)
  *sum = sm;
}

// ----------------------------------------------------------------------------- per-format groups

template <int FMT>
struct QGroup;

template <>
struct QGroup<NS_GGML_MXFP4> {
  static constexpr int kParts = 1;
  uint32_t q[4];
  float scale;  // 2^(e-128); cvt yields e2m1 values = GGML table / 2

  __device__ __forceinline__ void load(const uint8_t* row, int g) {
    uint32_t w[5];
    lds_words_unaligned<5>(row + 17 * g, w);
    scale = e8m0_half_scale(w[0] & 0xFFu);
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = __funnelshift_r(w[i], w[i + 1], 8);
  }
  // sub-chunk s: payload bytes 4s..4s+3 -> elements {4s+i, 16+4s+i}
  template <int NT, int XG = 32>
  static __device__ __forceinline__ void load_x(const float* x, int64_t xs, const int (&tok)[NT], int nt, int g,
                                                int s, float (&xv)[NT][8]) {
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      if (t < nt) {
        const float* p = x + tok[t] * xs + XG * g;
        float4 a = *reinterpret_cast<const float4*>(p + 4 * s);
        float4 b = *reinterpret_cast<const float4*>(p + 16 + 4 * s);
        xv[t][0] = a.x; xv[t][1] = b.x; xv[t][2] = a.y; xv[t][3] = b.y;
        xv[t][4] = a.z; xv[t][5] = b.z; xv[t][6] = a.w; xv[t][7] = b.w;
      }
    }
  }
  template <int NT>
  __device__ __forceinline__ void fma(int s, const float (&xv)[NT][8], int nt, float (&part)[NT][kParts]) const {
    uint32_t h[4];
    e2m1x4_to_f16x2(q[s], h);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = f16x2_to_float2(h[i]);
#pragma unroll
      for (int t = 0; t < NT; ++t)
        if (t < nt) part[t][0] = fmaf(xv[t][2 * i + 1], f.y, fmaf(xv[t][2 * i], f.x, part[t][0]));
    }
  }
  template <int NT>
  __device__ __forceinline__ void finish(const float (&part)[NT][kParts], const float (&)[NT], int nt,
                                         float (&acc)[NT]) const {
#pragma unroll
    for (int t = 0; t < NT; ++t)
      if (t < nt) acc[t] = fmaf(part[t][0] * 2.0f, scale, acc[t]);
  }
};

template <>
struct QGroup<NS_GGML_Q8_0> {
  static constexpr int kParts = 1;
  uint32_t q[8];
  float d;

  __device__ __forceinline__ void load(const uint8_t* row, int g) {
    uint32_t w[9];
    lds_words_unaligned<9>(row + 34 * g, w);
    d = f16_bits_to_float(w[0]);
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = __funnelshift_r(w[i], w[i + 1], 16) ^ 0x80808080u;
  }
  template <int NT, int XG = 32>
  static __device__ __forceinline__ void load_x(const float* x, int64_t xs, const int (&tok)[NT], int nt, int g,
                                                int s, float (&xv)[NT][8]) {
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      if (t < nt) {
        const float* p = x + tok[t] * xs + XG * g + 8 * s;
        float4 a = *reinterpret_cast<const float4*>(p);
        float4 b = *reinterpret_cast<const float4*>(p + 4);
        xv[t][0] = a.x; xv[t][1] = a.y; xv[t][2] = a.z; xv[t][3] = a.w;
        xv[t][4] = b.x; xv[t][5] = b.y; xv[t][6] = b.z; xv[t][7] = b.w;
      }
    }
  }
  template <int NT>
  __device__ __forceinline__ void fma(int s, const float (&xv)[NT][8], int nt, float (&part)[NT][kParts]) const {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float f = byte_as_float(q[2 * s + (j >> 2)], j & 3, k2p23 + 128.0f);  // int8 value
#pragma unroll
      for (int t = 0; t < NT; ++t)
        if (t < nt) part[t][0] = fmaf(xv[t][j], f, part[t][0]);
    }
  }
  template <int NT>
  __device__ __forceinline__ void finish(const float (&part)[NT][kParts], const float (&)[NT], int nt,
                                         float (&acc)[NT]) const {
#pragma unroll
    for (int t = 0; t < NT; ++t)
      if (t < nt) acc[t] = fmaf(part[t][0], d, acc[t]);
  }
};

template <>
struct QGroup<NS_GGML_Q4_K> {
  static constexpr int kParts = 1;
  uint32_t q[8];
  float dsc, mmn;  // d*sc and dmin*mn of this sub-block (both exact in fp32)

  // sub-block s's 6-bit scale and min from the 12 scale bytes (words h1, h2, h3 = bytes 0-3, 4-7,
  // 8-11): s < 4 reads bytes s and s + 4; s >= 4 combines byte s + 4 with the top bits of bytes
  // s - 4 and s.  Byte (s & 3) of each word, so no indexing by s.
  __device__ __forceinline__ void scales(uint32_t hdw, uint32_t h1, uint32_t h2, uint32_t h3, int s) {
    const unsigned sh = 8u * (unsigned)(s & 3);
    const uint32_t b1 = (h1 >> sh) & 0xFFu, b2 = (h2 >> sh) & 0xFFu, b3 = (h3 >> sh) & 0xFFu;
    const uint32_t sc = s < 4 ? (b1 & 63u) : ((b3 & 0x0Fu) | ((b1 >> 6) << 4));
    const uint32_t mn = s < 4 ? (b2 & 63u) : ((b3 >> 4) | ((b2 >> 6) << 4));
    dsc = f16_bits_to_float(hdw) * (float)sc;
    mmn = f16_bits_to_float(hdw >> 16) * (float)mn;
  }

  __device__ __forceinline__ void load(const uint8_t* row, int g) {
    const uint8_t* p = row + 144 * (g >> 3);
    const int s = g & 7;
    uint32_t hd[4];
    lds_words_unaligned<4>(p, hd);  // d | dmin | scales[0..11]
    scales(hd[0], hd[1], hd[2], hd[3], s);
    uint32_t w[8];
    lds_words_unaligned<8>(p + 16 + 32 * (s >> 1), w);
    const unsigned sh = (s & 1) ? 4u : 0u;
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = (w[i] >> sh) & 0x0F0F0F0Fu;
  }
  // the same from a 16-byte aligned row (superblocks are 144 = 9 x 16 bytes): three vector loads
  __device__ __forceinline__ void load_aligned(const uint8_t* row, int g) {
    const uint4* p = reinterpret_cast<const uint4*>(row + 144 * (g >> 3));
    const int s = g & 7;
    const uint4 hd = p[0];
    scales(hd.x, hd.y, hd.z, hd.w, s);
    const uint4 a = p[1 + 2 * (s >> 1)], b = p[2 + 2 * (s >> 1)];
    const unsigned sh = (s & 1) ? 4u : 0u;
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = (w[i] >> sh) & 0x0F0F0F0Fu;
  }
  template <int NT, int XG = 32>
  static __device__ __forceinline__ void load_x(const float* x, int64_t xs, const int (&tok)[NT], int nt, int g,
                                                int s, float (&xv)[NT][8]) {
    QGroup<NS_GGML_Q8_0>::load_x<NT, XG>(x, xs, tok, nt, g, s, xv);
  }
  template <int NT>
  __device__ __forceinline__ void fma(int s, const float (&xv)[NT][8], int nt, float (&part)[NT][kParts]) const {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float f = byte_as_float(q[2 * s + (j >> 2)], j & 3, k2p23);
#pragma unroll
      for (int t = 0; t < NT; ++t)
        if (t < nt) part[t][0] = fmaf(xv[t][j], f, part[t][0]);
    }
  }
  template <int NT>
  __device__ __forceinline__ void finish(const float (&part)[NT][kParts], const float (&xsum)[NT], int nt,
                                         float (&acc)[NT]) const {
#pragma unroll
    for (int t = 0; t < NT; ++t)
      if (t < nt) acc[t] = fmaf(-mmn, xsum[t], fmaf(part[t][0], dsc, acc[t]));
  }
};

template <>
struct QGroup<NS_GGML_Q5_K> {
  static constexpr int kParts = 1;
  uint32_t q[8];  // 5-bit codes 0..31, one per byte
  float dsc, mmn;

  // neurostream/compute/quant.py:59-81: d*sc*q - dmin*mn with q = nibble + 16 * (qh bit)
  __device__ __forceinline__ void load(const uint8_t* row, int g) {
    const uint8_t* p = row + 176 * (g >> 3);
    const int s = g & 7;
    uint32_t hd[4];
    lds_words_unaligned<4>(p, hd);  // d | dmin | scales[0..11]
    QGroup<NS_GGML_Q4_K> k4;
    k4.scales(hd[0], hd[1], hd[2], hd[3], s);
    dsc = k4.dsc;
    mmn = k4.mmn;
    uint32_t w[8], h[8];
    lds_words_unaligned<8>(p + 48 + 32 * (s >> 1), w);
    lds_words_unaligned<8>(p + 16, h);
    const unsigned sh = (s & 1) ? 4u : 0u;
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = ((w[i] >> sh) & 0x0F0F0F0Fu) | (((h[i] >> (unsigned)s) & 0x01010101u) << 4);
  }
  template <int NT, int XG = 32>
  static __device__ __forceinline__ void load_x(const float* x, int64_t xs, const int (&tok)[NT], int nt, int g,
                                                int s, float (&xv)[NT][8]) {
    QGroup<NS_GGML_Q8_0>::load_x<NT, XG>(x, xs, tok, nt, g, s, xv);
  }
  template <int NT>
  __device__ __forceinline__ void fma(int s, const float (&xv)[NT][8], int nt, float (&part)[NT][kParts]) const {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float f = byte_as_float(q[2 * s + (j >> 2)], j & 3, k2p23);
#pragma unroll
      for (int t = 0; t < NT; ++t)
        if (t < nt) part[t][0] = fmaf(xv[t][j], f, part[t][0]);
    }
  }
  template <int NT>
  __device__ __forceinline__ void finish(const float (&part)[NT][kParts], const float (&xsum)[NT], int nt,
                                         float (&acc)[NT]) const {
#pragma unroll
    for (int t = 0; t < NT; ++t)
      if (t < nt) acc[t] = fmaf(-mmn, xsum[t], fmaf(part[t][0], dsc, acc[t]));
  }
};

template <>
struct QGroup<NS_GGML_Q4_0> {
  static constexpr int kParts = 1;
  uint32_t q[4];  // payload bytes 0..15
  float d;

  // neurostream/compute/quant.py:118-126: d * (nibble - 8)
  __device__ __forceinline__ void load(const uint8_t* row, int g) {
    uint32_t w[5];
    lds_words_unaligned<5>(row + 18 * g, w);
    d = f16_bits_to_float(w[0]);
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = __funnelshift_r(w[i], w[i + 1], 16);
  }
  // sub-chunk s: payload bytes 4s..4s+3 -> elements {4s+i, 16+4s+i} (the MXFP4 pairing)
  template <int NT, int XG = 32>
  static __device__ __forceinline__ void load_x(const float* x, int64_t xs, const int (&tok)[NT], int nt, int g,
                                                int s, float (&xv)[NT][8]) {
    QGroup<NS_GGML_MXFP4>::load_x<NT, XG>(x, xs, tok, nt, g, s, xv);
  }
  template <int NT>
  __device__ __forceinline__ void fma(int s, const float (&xv)[NT][8], int nt, float (&part)[NT][kParts]) const {
    const uint32_t lo = q[s] & 0x0F0F0F0Fu, hi = (q[s] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float fl = byte_as_float(lo, i, k2p23 + 8.0f), fh = byte_as_float(hi, i, k2p23 + 8.0f);
#pragma unroll
      for (int t = 0; t < NT; ++t)
        if (t < nt) part[t][0] = fmaf(xv[t][2 * i + 1], fh, fmaf(xv[t][2 * i], fl, part[t][0]));
    }
  }
  template <int NT>
  __device__ __forceinline__ void finish(const float (&part)[NT][kParts], const float (&)[NT], int nt,
                                         float (&acc)[NT]) const {
#pragma unroll
    for (int t = 0; t < NT; ++t)
      if (t < nt) acc[t] = fmaf(part[t][0], d, acc[t]);
  }
};

template <>
struct QGroup<NS_GGML_Q6_K> {
  static constexpr int kParts = 2;  // elements 0..15 and 16..31 have their own scale
  uint32_t q[8];
  float dsc0, dsc1;

  __device__ __forceinline__ void load(const uint8_t* row, int g) {
    const uint8_t* p = row + 210 * (g >> 3);
    const int h = (g >> 2) & 1, i = g & 3;
    uint32_t ql[8], qh[8];
    lds_words_unaligned<8>(p + 64 * h + 32 * (i & 1), ql);
    lds_words_unaligned<8>(p + 128 + 32 * h, qh);
    const unsigned lsh = (i >> 1) ? 4u : 0u, hsh = 2u * (unsigned)i;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint32_t lo = (ql[j] >> lsh) & 0x0F0F0F0Fu;
      uint32_t hi = ((qh[j] >> hsh) & 0x03030303u) << 4;
      q[j] = lo | hi;  // 6-bit q per byte
    }
    const uint32_t scw = lds_u32_unaligned(p + 192 + 8 * h + 2 * i);  // bytes sc[2i], sc[2i+1]
    const uint32_t dw = lds_u32_unaligned(p + 208);
    const float d = f16_bits_to_float(dw);
    dsc0 = d * (float)(int8_t)(scw & 0xFFu);
    dsc1 = d * (float)(int8_t)((scw >> 8) & 0xFFu);
  }
  template <int NT, int XG = 32>
  static __device__ __forceinline__ void load_x(const float* x, int64_t xs, const int (&tok)[NT], int nt, int g,
                                                int s, float (&xv)[NT][8]) {
    QGroup<NS_GGML_Q8_0>::load_x<NT, XG>(x, xs, tok, nt, g, s, xv);
  }
  template <int NT>
  __device__ __forceinline__ void fma(int s, const float (&xv)[NT][8], int nt, float (&part)[NT][kParts]) const {
    const int pi = s >> 1;  // sub-chunks 0,1 -> scale 0; 2,3 -> scale 1
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float f = byte_as_float(q[2 * s + (j >> 2)], j & 3, k2p23 + 32.0f);  // q - 32
#pragma unroll
      for (int t = 0; t < NT; ++t)
        if (t < nt) part[t][pi] = fmaf(xv[t][j], f, part[t][pi]);
    }
  }
  template <int NT>
  __device__ __forceinline__ void finish(const float (&part)[NT][kParts], const float (&)[NT], int nt,
                                         float (&acc)[NT]) const {
#pragma unroll
    for (int t = 0; t < NT; ++t)
      if (t < nt) acc[t] = fmaf(part[t][1], dsc1, fmaf(part[t][0], dsc0, acc[t]));
  }
};

// ----------------------------------------------------------------------------- row dots

// acc[r][t] += sum over this lane's groups of row r (smem) . x[t]
// rows[r] may be nullptr (row absent) for r >= nrows; nrows is warp-uniform.
// x: generic pointer; token t's activations are the row x + tok[t]*xs (floats,
// 16-byte aligned rows), group g of it at + XG*g, for t < nt <= NT.  In shared
// memory XG = 36 keeps the lanes (one group each) on distinct banks.
// Groups g0, g0 + gstep, .. (gstep = 32: one lane per group of the row).  ALL: every one of the
// R rows and NT tokens is valid (no per-element tests); otherwise rows >= nrows and tokens >= nt
// are skipped.
template <int FMT, int NT, int R, int XG = 32, bool ALL = false>
__device__ __forceinline__ void dot_rows(const uint8_t* const (&rows)[R], int nrows_, int ngroups, int g0,
                                         const float* x, int64_t xs, const int (&tok)[NT], int nt_,
                                         float (&acc)[R][NT], int gstep = 32) {
  using G = QGroup<FMT>;
  const int nrows = ALL ? R : nrows_, nt = ALL ? NT : nt_;
  for (int g = g0; g < ngroups; g += gstep) {
    G q[R];
#pragma unroll
    for (int r = 0; r < R; ++r)
      if (r < nrows) q[r].load(rows[r], g);
    float part[R][NT][G::kParts];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int p = 0; p < G::kParts; ++p) part[r][t][p] = 0.f;
    float xsum[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) xsum[t] = 0.f;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      float xv[NT][8];
      G::template load_x<NT, XG>(x, xs, tok, nt, g, s, xv);
      if (FMT == NS_GGML_Q4_K || FMT == NS_GGML_Q5_K) {
#pragma unroll
        for (int t = 0; t < NT; ++t)
          if (t < nt)
            xsum[t] += ((xv[t][0] + xv[t][1]) + (xv[t][2] + xv[t][3])) + ((xv[t][4] + xv[t][5]) + (xv[t][6] + xv[t][7]));
      }
#pragma unroll
      for (int r = 0; r < R; ++r)
        if (r < nrows) q[r].template fma<NT>(s, xv, nt, part[r]);
    }
#pragma unroll
    for (int r = 0; r < R; ++r)
      if (r < nrows) q[r].template finish<NT>(part[r], xsum, nt, acc[r]);
  }
}

}  // namespace ns
