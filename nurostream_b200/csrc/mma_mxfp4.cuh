// MXFP4 dot products on the tensor cores (mma.sync m16n8k16, f16 in, f32 accumulate).
//
// Roles: the B operand (16 k x 8 n) is EIGHT WEIGHT ROWS, decoded straight from
// the GGUF bytes staged in shared memory: cvt.rn.f16x2.e2m1x2 turns one payload
// byte (two e2m1 codes) into one f16x2 B register, exactly.  The A operand
// (16 rows x 16 k) holds the activations: row 2i+p is part p (0 = high, 1 =
// low) of token i, where a token vector v is scaled by 2^sigma and split as
// hi = f16(v*2^sigma), lo = f16(v*2^sigma - hi).  Every product of an e2m1
// value (2 significant bits) with an 11-bit part is exact in fp32, so the MMA
// computes sum(w*v) with fp32 accumulation and ~22 bits of each activation.
//
// k mapping: a 32-element block is two MMAs (s = 0, 1).  Lane (g, q) (g = lane/4,
// q = lane%4) supplies weight row g's payload word q (bytes 4q..4q+3); byte
// 4q+2s feeds k-pair q and byte 4q+2s+1 feeds k-pair q+4 of MMA s.  A k-pair of
// byte j is the element pair (j, j+16) -- the low and high nibble -- so the
// A fragments carry v[j], v[j+16] in the same order (see build_xfrag).
//
// D: lane (g, q) ends with (x-part g, weight rows 2q and 2q+1) in c0/c1 and
// (x-part g+8, same rows) in c2/c3.  The per-block E8M0 scale of each weight
// row is applied to D after the block's two MMAs.
#pragma once

#include "common.cuh"

namespace ns {

__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// One payload word (4 bytes, 8 e2m1 codes) -> the four B registers of the
// block's two MMAs: {s0 k-pair q, s0 k-pair q+4, s1 k-pair q, s1 k-pair q+4}.
__device__ __forceinline__ void e2m1_word_to_b(uint32_t w, uint32_t (&b)[4]) {
  asm("{\n .reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %4;\n"
      " cvt.rn.f16x2.e2m1x2 %0, b0;\n cvt.rn.f16x2.e2m1x2 %1, b1;\n"
      " cvt.rn.f16x2.e2m1x2 %2, b2;\n cvt.rn.f16x2.e2m1x2 %3, b3;\n}"
      : "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3])
      : "r"(w));
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Exponent sigma such that max|v| * 2^sigma lies in [2^13, 2^14): the hi part
// then stays well inside fp16 range.  The doubled GGML e2m1 table (cvt yields
// table/2) is folded in by the +1 of the output factor 2^(1 - sigma).
__device__ __forceinline__ int xsplit_sigma(float vmax) {
  if (!(vmax > 0.f) || !isfinite(vmax)) return 0;
  int e;
  frexpf(vmax, &e);  // vmax = m * 2^e, m in [0.5, 1)
  int s = 14 - e;
  return s > 100 ? 100 : (s < -100 ? -100 : s);
}

// Fragment image of one token vector: xf[p][b][q] = 4 u32, p = part.
//   u32 0: (v[32b+4q],   v[32b+4q+16])    MMA s=0, k-pair q
//   u32 1: (v[32b+4q+1], v[32b+4q+17])    MMA s=0, k-pair q+4
//   u32 2: (v[32b+4q+2], v[32b+4q+18])    MMA s=1, k-pair q
//   u32 3: (v[32b+4q+3], v[32b+4q+19])    MMA s=1, k-pair q+4
// Layout in shared memory: part stride = nblocks*64 + 64 bytes (padding keeps
// the hi and lo images of one (b, q) in different banks).
__device__ __forceinline__ int xfrag_part_stride_u4(int nblocks) { return nblocks * 4 + 4; }
__device__ __forceinline__ int xfrag_vec_u4(int nblocks) { return 2 * xfrag_part_stride_u4(nblocks); }

// Build the image of v (fp32, length 32*nblocks, generic pointer) with scale 2^sigma.
// Called by `nthr` threads with index `tid` (cooperative).
__device__ __forceinline__ void build_xfrag(const float* v, int nblocks, int sigma, uint4* img, int tid, int nthr) {
  const float sc = ldexpf(1.0f, sigma);
  const int ps = xfrag_part_stride_u4(nblocks);
  for (int i = tid; i < nblocks * 4; i += nthr) {
    const int b = i >> 2, q = i & 3;
    const float* p = v + 32 * b + 4 * q;
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float x0 = p[j] * sc, x1 = p[j + 16] * sc;
      __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
      float r0 = x0 - __half2float(h0), r1 = x1 - __half2float(h1);
      __half2 hh = __halves2half2(h0, h1);
      hi[j] = *reinterpret_cast<uint32_t*>(&hh);
      lo[j] = pack_f16x2(r0, r1);
    }
    img[b * 4 + q] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    img[ps + b * 4 + q] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  }
}

// E8M0 half scale 2^(e-128) of every (row, block) of a staged tile, block-major:
// sc[b * rows_pad + r].  Exact for every e (0 and 1 give fp32 subnormals).
__device__ __forceinline__ void mxfp4_scales(const uint8_t* const* rowp, int nrows, int nblocks, int rows_pad,
                                             float* sc, int tid, int nthr) {
  for (int i = tid; i < nrows * nblocks; i += nthr) {
    const int r = i / nblocks, b = i - r * nblocks;
    sc[b * rows_pad + r] = e8m0_half_scale(rowp[r][17 * b]);
  }
}

// Partial sums of one 8-row group over blocks [b0, b1):
//   acc[0] (x-part g,   row 2q), acc[1] (x-part g,   row 2q+1),
//   acc[2] (x-part g+8, row 2q), acc[3] (x-part g+8, row 2q+1).
// row_g: shared-memory address of this lane's weight row g (rows of the group
// beyond the tile point at a valid row; their results are discarded).
// xf0/xf1: image rows for x-part g and g+8 (nullptr -> zeros).
// sc: scale array (block-major, rows_pad per block), grp_row0 = first row of the group.
__device__ __forceinline__ void mxfp4_group_mma(const uint8_t* row_g, const uint4* xf0, const uint4* xf1, int b0,
                                                int b1, int q, const float* sc, int rows_pad, int grp_row0,
                                                float (&acc)[4]) {
  const uint8_t* pw = row_g + 1 + 4 * q;   // payload word q of block 0
  const float* scr = sc + grp_row0 + 2 * q;
#pragma unroll 2
  for (int b = b0; b < b1; ++b) {
    const uint32_t w = lds_u32_unaligned(pw + 17 * b);
    uint32_t bw[4];
    e2m1_word_to_b(w, bw);
    uint4 x0 = xf0 ? xf0[b * 4 + q] : make_uint4(0, 0, 0, 0);
    uint4 x1 = xf1 ? xf1[b * 4 + q] : make_uint4(0, 0, 0, 0);
    // A regs: {row g k-pair q, row g+8 k-pair q, row g k-pair q+4, row g+8 k-pair q+4}
    const uint32_t a0[4] = {x0.x, x1.x, x0.y, x1.y};
    const uint32_t a1[4] = {x0.z, x1.z, x0.w, x1.w};
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    mma_f16_16816(d, a0, bw[0], bw[1]);
    mma_f16_16816(d, a1, bw[2], bw[3]);
    const float2 s = *reinterpret_cast<const float2*>(scr + b * rows_pad);
    acc[0] = fmaf(d[0], s.x, acc[0]);
    acc[1] = fmaf(d[1], s.y, acc[1]);
    acc[2] = fmaf(d[2], s.x, acc[2]);
    acc[3] = fmaf(d[3], s.y, acc[3]);
  }
}

}  // namespace ns
