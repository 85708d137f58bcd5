// ns_dequant: GGML bytes -> floats, bit-exact with the reference decoders
// (neurostream/compute/quant.py:24-184).  One thread per block; products are
// formed in the reference's order with explicit round-to-nearest intrinsics so
// that no FMA contraction can change a bit.
#include "common.cuh"

namespace ns {

__device__ __forceinline__ uint32_t ld_u8(const uint8_t* p, int64_t i) { return p[i]; }
__device__ __forceinline__ uint32_t ld_u16le(const uint8_t* p, int64_t i) { return p[i] | (p[i + 1] << 8); }

// GGML's MXFP4 code table (e2m1 doubled), +0 for the negative-zero code.
__device__ __constant__ float c_mxfp4_values[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};

template <int FMT>
__device__ __forceinline__ void decode_block(const uint8_t* b, float (&v)[256]);

template <>
__device__ __forceinline__ void decode_block<NS_GGML_MXFP4>(const uint8_t* b, float (&v)[256]) {
  const float scale = e8m0_half_scale(b[0]);
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    uint32_t q = b[1 + j];
    v[j] = __fmul_rn(scale, c_mxfp4_values[q & 15]);
    v[j + 16] = __fmul_rn(scale, c_mxfp4_values[q >> 4]);
  }
}

template <>
__device__ __forceinline__ void decode_block<NS_GGML_Q8_0>(const uint8_t* b, float (&v)[256]) {
  const float d = f16_bits_to_float(ld_u16le(b, 0));
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __fmul_rn(d, (float)(int8_t)b[2 + j]);
}

template <>
__device__ __forceinline__ void decode_block<NS_GGML_Q4_0>(const uint8_t* b, float (&v)[256]) {
  const float d = f16_bits_to_float(ld_u16le(b, 0));
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    uint32_t q = b[2 + j];
    v[j] = __fmul_rn(d, (float)((int)(q & 15) - 8));
    v[j + 16] = __fmul_rn(d, (float)((int)(q >> 4) - 8));
  }
}

// get_scale_min_k4 for sub-block s (Q4_K / Q5_K scale bytes at sc[0..11]).
__device__ __forceinline__ void k_scale_min(const uint8_t* sc, int s, float* scale, float* mn) {
  uint32_t a, m;
  if (s < 4) {
    a = sc[s] & 63u;
    m = sc[s + 4] & 63u;
  } else {
    a = (sc[s + 4] & 0x0Fu) | ((sc[s - 4] >> 6) << 4);
    m = (sc[s + 4] >> 4) | ((sc[s] >> 6) << 4);
  }
  *scale = (float)a;
  *mn = (float)m;
}

template <>
__device__ __forceinline__ void decode_block<NS_GGML_Q4_K>(const uint8_t* b, float (&v)[256]) {
  const float d = f16_bits_to_float(ld_u16le(b, 0)), dmin = f16_bits_to_float(ld_u16le(b, 2));
#pragma unroll 1
  for (int s = 0; s < 8; ++s) {
    float sc, mn;
    k_scale_min(b + 4, s, &sc, &mn);
    const float scale = __fmul_rn(d, sc), off = __fmul_rn(dmin, mn);
    const uint8_t* qs = b + 16 + 32 * (s >> 1);
    const int sh = (s & 1) * 4;
#pragma unroll
    for (int l = 0; l < 32; ++l) v[32 * s + l] = __fsub_rn(__fmul_rn(scale, (float)((qs[l] >> sh) & 15)), off);
  }
}

template <>
__device__ __forceinline__ void decode_block<NS_GGML_Q5_K>(const uint8_t* b, float (&v)[256]) {
  const float d = f16_bits_to_float(ld_u16le(b, 0)), dmin = f16_bits_to_float(ld_u16le(b, 2));
  const uint8_t* qh = b + 16;
#pragma unroll 1
  for (int s = 0; s < 8; ++s) {
    float sc, mn;
    k_scale_min(b + 4, s, &sc, &mn);
    const float scale = __fmul_rn(d, sc), off = __fmul_rn(dmin, mn);
    const uint8_t* qs = b + 48 + 32 * (s >> 1);
    const int sh = (s & 1) * 4;
#pragma unroll
    for (int l = 0; l < 32; ++l) {
      int q = ((qs[l] >> sh) & 15) + (((qh[l] >> s) & 1) << 4);
      v[32 * s + l] = __fsub_rn(__fmul_rn(scale, (float)q), off);
    }
  }
}

template <>
__device__ __forceinline__ void decode_block<NS_GGML_Q6_K>(const uint8_t* b, float (&v)[256]) {
  const float d = f16_bits_to_float(ld_u16le(b, 208));
#pragma unroll 1
  for (int h = 0; h < 2; ++h) {
    const uint8_t* ql = b + 64 * h;
    const uint8_t* qh = b + 128 + 32 * h;
    const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192 + 8 * h);
#pragma unroll 1
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int l = 0; l < 32; ++l) {
        int lo = (ql[(i & 1) * 32 + l] >> ((i >> 1) * 4)) & 15;
        int hi = (qh[l] >> (2 * i)) & 3;
        int q = (lo | (hi << 4)) - 32;
        float ds = __fmul_rn(d, (float)sc[(l >> 4) + 2 * i]);
        v[128 * h + 32 * i + l] = __fmul_rn(ds, (float)q);
      }
    }
  }
}

template <int FMT, int BE, int BB>
__global__ void dequant_kernel(const uint8_t* raw, int64_t nblocks, int64_t n_elements, void* out, int out_dtype) {
  int64_t blk = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (blk >= nblocks) return;
  float v[256];
  decode_block<FMT>(raw + blk * BB, v);
  const int64_t e0 = blk * BE;
#pragma unroll 4
  for (int j = 0; j < BE; ++j)
    if (e0 + j < n_elements) store_float(out, out_dtype, e0 + j, v[j]);
}

__global__ void float_convert_kernel(const uint8_t* raw, int src, int64_t n, void* out, int out_dtype) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float v;
  if (src == NS_GGML_F32) v = reinterpret_cast<const float*>(raw)[i];
  else if (src == NS_GGML_F16) v = f16_bits_to_float(ld_u16le(raw, 2 * i));
  else v = __uint_as_float(ld_u16le(raw, 2 * i) << 16);
  store_float(out, out_dtype, i, v);
}

template <int FMT, int BE, int BB>
static int launch_dequant(const uint8_t* raw, int64_t nblocks, int64_t n, void* out, int od, cudaStream_t s) {
  const int threads = 128;
  int64_t grid = (nblocks + threads - 1) / threads;
  dequant_kernel<FMT, BE, BB><<<(unsigned)grid, threads, 0, s>>>(raw, nblocks, n, out, od);
  NS_CUDA_TRY(cudaGetLastError());
  return NS_OK;
}

}  // namespace ns

extern "C" int ns_dequant(const uint8_t* raw, size_t raw_bytes, int ggml_type, int64_t n_elements, void* out,
                          int out_dtype, ns_stream_t stream) {
  using namespace ns;
  int be, bb;
  if (!block_layout(ggml_type, &be, &bb))
    return fail(NS_ERR_UNSUPPORTED, "ns_dequant: no dequant kernel for ggml type %d", ggml_type);
  if (!float_type_ok(out_dtype)) return fail(NS_ERR_INVALID, "ns_dequant: bad output type %d", out_dtype);
  if (n_elements < 0) return fail(NS_ERR_INVALID, "ns_dequant: negative element count");
  if (n_elements == 0) return NS_OK;
  if (!raw || !out) return fail(NS_ERR_INVALID, "ns_dequant: null pointer");
  const int64_t nblocks_avail = (int64_t)(raw_bytes / bb);
  const int64_t nblocks = (n_elements + be - 1) / be;
  if (nblocks > nblocks_avail)
    return fail(NS_ERR_SIZE, "ns_dequant: %lld elements need %lld blocks, buffer holds %lld",
                (long long)n_elements, (long long)nblocks, (long long)nblocks_avail);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (ggml_type) {
    case NS_GGML_F32:
    case NS_GGML_F16:
    case NS_GGML_BF16: {
      float_convert_kernel<<<(unsigned)((n_elements + 255) / 256), 256, 0, s>>>(raw, ggml_type, n_elements, out,
                                                                               out_dtype);
      NS_CUDA_TRY(cudaGetLastError());
      return NS_OK;
    }
    case NS_GGML_MXFP4: return launch_dequant<NS_GGML_MXFP4, 32, 17>(raw, nblocks, n_elements, out, out_dtype, s);
    case NS_GGML_Q8_0: return launch_dequant<NS_GGML_Q8_0, 32, 34>(raw, nblocks, n_elements, out, out_dtype, s);
    case NS_GGML_Q4_0: return launch_dequant<NS_GGML_Q4_0, 32, 18>(raw, nblocks, n_elements, out, out_dtype, s);
    case NS_GGML_Q4_K: return launch_dequant<NS_GGML_Q4_K, 256, 144>(raw, nblocks, n_elements, out, out_dtype, s);
    case NS_GGML_Q5_K: return launch_dequant<NS_GGML_Q5_K, 256, 176>(raw, nblocks, n_elements, out, out_dtype, s);
    default: return launch_dequant<NS_GGML_Q6_K, 256, 210>(raw, nblocks, n_elements, out, out_dtype, s);
  }
}
