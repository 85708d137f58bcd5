// ns_synth_fill: device twin of nurostream_b200/synth.py (seeded synthetic
// GGUF tensors).  splitmix64 (Steele, Lea & Flood 2014) over a per-stream key;
// see the Python module for the distributions.  Integer work plus one fp32
// multiply and one fp16/bf16 rounding per value, so host and device agree bit
// for bit.
#include "common.cuh"

namespace ns {

constexpr uint64_t kGamma = 0x9E3779B97F4A7C15ull;
constexpr uint64_t kAuxSalt = 0xA5A5A5A5A5A5A5A5ull;
constexpr uint64_t kStreamSalt = 0x632BE59BD9B4E019ull;

__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z ^= z >> 30;
  z *= 0xBF58476D1CE4E5B9ull;
  z ^= z >> 27;
  z *= 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__host__ __device__ __forceinline__ uint64_t stream_key(uint64_t seed, uint64_t stream) {
  return mix64((seed * kGamma) ^ (stream + kStreamSalt));
}

__device__ __forceinline__ uint64_t word_at(uint64_t key, uint64_t i) { return mix64(key + (i + 1) * kGamma); }

__device__ __forceinline__ uint32_t scale_fp16_bits(uint64_t key, uint64_t idx, float mult) {
  uint64_t w = word_at(key ^ kAuxSalt, idx);
  float v = __fmul_rn((float)(0.5 + (double)(w >> 41) * 0x1p-23), mult);  // 0.5+u exact in fp32
  return __half_as_ushort(__float2half_rn(v));
}

// One thread per output byte group of 8 (word-aligned within the stream).
__global__ void synth_quant_kernel(uint8_t* dst, uint64_t count, uint64_t start, uint64_t key, int bb, int fmt,
                                   int e_lo, int e_hi, float mult) {
  uint64_t wi = (start >> 3) + (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;  // stream word index
  uint64_t p0 = wi << 3;
  if (p0 >= start + count) return;
  uint64_t w = word_at(key, wi);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    uint64_t p = p0 + j;
    if (p < start || p >= start + count) continue;
    uint32_t byte = (uint32_t)(w >> (8 * j)) & 0xFFu;
    uint64_t off = p % (uint64_t)bb, blk = p / (uint64_t)bb;
    if (fmt == NS_GGML_MXFP4) {
      if (off == 0) byte = (uint32_t)e_lo + byte % (uint32_t)(e_hi - e_lo + 1);
    } else {
      int field = -1;
      uint64_t f0 = 0;
      if (fmt == NS_GGML_Q6_K) {
        if (off == 208 || off == 209) { field = 0; f0 = 208; }
      } else if (off < 2) {
        field = 0; f0 = 0;
      } else if ((fmt == NS_GGML_Q4_K || fmt == NS_GGML_Q5_K) && off < 4) {
        field = 1; f0 = 2;
      }
      if (field >= 0) {
        uint32_t h = scale_fp16_bits(key, blk * 2 + field, mult);
        byte = (off == f0) ? (h & 0xFFu) : (h >> 8);
      }
    }
    dst[p - start] = (uint8_t)byte;
  }
}

__global__ void synth_float_kernel(void* dst, uint64_t count, uint64_t start, uint64_t key, float sigma, int bf16) {
  uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= count) return;
  uint64_t base = 12 * (start + i);
  int64_t s = 0;
#pragma unroll
  for (int j = 0; j < 12; ++j) s += (int64_t)(word_at(key, base + j) >> 40);
  float v = __fmul_rn(__double2float_rn((double)s * 0x1p-24 - 6.0), sigma);
  if (bf16) reinterpret_cast<__nv_bfloat16*>(dst)[i] = __float2bfloat16_rn(v);
  else reinterpret_cast<float*>(dst)[i] = v;
}

}  // namespace ns

extern "C" int ns_synth_fill(void* dst, uint64_t count, int kind, uint64_t seed, uint64_t stream, uint64_t start,
                             float sigma, int e_lo, int e_hi, float scale_mult, ns_stream_t s) {
  using namespace ns;
  if (count == 0) return NS_OK;
  if (!dst) return fail(NS_ERR_INVALID, "ns_synth_fill: null destination");
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(s);
  const uint64_t key = stream_key(seed, stream);
  if (kind == NS_SYNTH_F32 || kind == NS_SYNTH_BF16) {
    uint64_t grid = (count + 255) / 256;
    synth_float_kernel<<<(unsigned)grid, 256, 0, cs>>>(dst, count, start, key, sigma, kind == NS_SYNTH_BF16);
    NS_CUDA_TRY(cudaGetLastError());
    return NS_OK;
  }
  int be, bb;
  if (!block_layout(kind, &be, &bb) || be == 1)
    return fail(NS_ERR_UNSUPPORTED, "ns_synth_fill: no generator for kind %d", kind);
  if (kind == NS_GGML_MXFP4 && !(0 <= e_lo && e_lo <= e_hi && e_hi <= 255))
    return fail(NS_ERR_INVALID, "ns_synth_fill: bad exponent range %d..%d", e_lo, e_hi);
  uint64_t words = ((start + count + 7) >> 3) - (start >> 3);
  uint64_t grid = (words + 255) / 256;
  if (grid > 0x7FFFFFFFull) return fail(NS_ERR_INVALID, "ns_synth_fill: count too large for one call");
  synth_quant_kernel<<<(unsigned)grid, 256, 0, cs>>>(reinterpret_cast<uint8_t*>(dst), count, start, key, bb, kind,
                                                      e_lo, e_hi, scale_mult);
  NS_CUDA_TRY(cudaGetLastError());
  return NS_OK;
}
