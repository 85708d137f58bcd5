// Shared device/host helpers for the ns_b200 kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>

#include <algorithm>

#include "../../include/ns_b200.h"

namespace ns {

// ----------------------------------------------------------------------------- host errors

void set_error(const char* fmt, ...);                 // abi.cu
int fail(int status, const char* fmt, ...);           // sets message, returns status
int cuda_fail(cudaError_t e, const char* what);       // NS_ERR_CUDA with CUDA's message
int num_sms(int* out);                                // SM count of the current device (cached)

#define NS_CUDA_TRY(call)                                 \
  do {                                                    \
    cudaError_t _e = (call);                              \
    if (_e != cudaSuccess) return ::ns::cuda_fail(_e, #call); \
  } while (0)

inline bool block_layout(int t, int* be, int* bb) {
  switch (t) {
    case NS_GGML_F32: *be = 1; *bb = 4; return true;
    case NS_GGML_F16: *be = 1; *bb = 2; return true;
    case NS_GGML_BF16: *be = 1; *bb = 2; return true;
    case NS_GGML_MXFP4: *be = 32; *bb = 17; return true;
    case NS_GGML_Q4_0: *be = 32; *bb = 18; return true;
    case NS_GGML_Q8_0: *be = 32; *bb = 34; return true;
    case NS_GGML_Q4_K: *be = 256; *bb = 144; return true;
    case NS_GGML_Q5_K: *be = 256; *bb = 176; return true;
    case NS_GGML_Q6_K: *be = 256; *bb = 210; return true;
    default: return false;
  }
}

// Row bytes of K elements, or -1 if K is not a whole number of blocks.
inline int64_t row_bytes_of(int t, int64_t K) {
  int be, bb;
  if (!block_layout(t, &be, &bb) || K % be) return -1;
  return K / be * bb;
}

inline bool float_type_ok(int d) { return d == NS_F32 || d == NS_F16 || d == NS_BF16; }
inline int float_size(int d) { return d == NS_F32 ? 4 : 2; }

// ----------------------------------------------------------------------------- device error word

// One error word per device (a __device__ variable has one instance per device
// that loads the module).  Kernels OR bits into it; ns_device_error reads it.
// Defined here because the library is a single translation unit (ns_b200.cu).
__device__ unsigned int g_device_error = 0;

__device__ __forceinline__ void raise_device_error(unsigned bits) { atomicOr(&g_device_error, bits); }

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Upper bound of any device-side wait (a grid barrier, a bulk-copy completion).
constexpr uint64_t kWaitLimitNs = 1000000000ull;

// ----------------------------------------------------------------------------- float conversions

__device__ __forceinline__ float load_float(const void* p, int dtype, int64_t i) {
  if (dtype == NS_F32) return reinterpret_cast<const float*>(p)[i];
  if (dtype == NS_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}

// N values out[u] = p[idx(u)] (0 where idx(u) < 0) of a float tensor of type dtype, with the
// type switch outside the loads so that all N loads are in flight together.  (load_float in an
// unrolled loop converts each value right after its load, inside the type branch, which makes
// every load wait for the one before it.)
template <int N, typename IdxFn>
__device__ __forceinline__ void load_floats(const void* p, int dtype, IdxFn idx, float (&out)[N]) {
  if (dtype == NS_F32) {
    const float* f = static_cast<const float*>(p);
#pragma unroll
    for (int u = 0; u < N; ++u) {
      const int64_t i = idx(u);
      out[u] = i >= 0 ? f[i] : 0.f;
    }
  } else {
    const unsigned short* h = static_cast<const unsigned short*>(p);
    uint32_t r[N];
#pragma unroll
    for (int u = 0; u < N; ++u) {
      const int64_t i = idx(u);
      r[u] = i >= 0 ? (uint32_t)h[i] : 0u;
    }
    if (dtype == NS_F16) {
#pragma unroll
      for (int u = 0; u < N; ++u) out[u] = __half2float(__ushort_as_half((unsigned short)r[u]));
    } else {
#pragma unroll
      for (int u = 0; u < N; ++u) out[u] = __uint_as_float(r[u] << 16);  // bf16 -> fp32, exact
    }
  }
}

__device__ __forceinline__ void store_float(void* p, int dtype, int64_t i, float v) {
  if (dtype == NS_F32) reinterpret_cast<float*>(p)[i] = v;
  else if (dtype == NS_F16) reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  else reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}

__device__ __forceinline__ float f16_bits_to_float(uint32_t h) {
  return __half2float(__ushort_as_half((unsigned short)(h & 0xFFFFu)));
}

// GGML's E8M0 "half" scale 2^(e-128): e = 0, 1 are fp32 subnormals, 255 is 2^127.
__device__ __forceinline__ float e8m0_half_scale(uint32_t e) {
  return __uint_as_float(e < 2u ? (0x00200000u << e) : ((e - 1u) << 23));
}

// ----------------------------------------------------------------------------- smem byte access

// 32-bit word at a 4-byte aligned shared-memory address (a shared-window address, so the load is
// an ld.shared: a generic pointer rebuilt from an integer would be a generic load).
__device__ __forceinline__ uint32_t lds32(uint32_t saddr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(saddr));
  return v;
}

__device__ __forceinline__ void sts32(uint32_t saddr, uint32_t v) {
  asm volatile("st.shared.u32 [%0], %1;" ::"r"(saddr), "r"(v) : "memory");
}
__device__ __forceinline__ void sts128(uint32_t saddr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(saddr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// 32-bit little-endian word at an arbitrary byte address of shared memory.
__device__ __forceinline__ uint32_t lds_u32_unaligned(const uint8_t* p) {
  uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  uint32_t lo = w[0], hi = w[1];
  return __funnelshift_r(lo, hi, (unsigned)(a & 3) * 8u);
}

// n consecutive words starting at an arbitrary byte address (n aligned loads + n-1.. shifts).
template <int N>
__device__ __forceinline__ void lds_words_unaligned(const uint8_t* p, uint32_t (&out)[N]) {
  uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  unsigned sh = (unsigned)(a & 3) * 8u;
  uint32_t prev = w[0];
#pragma unroll
  for (int i = 0; i < N; ++i) {
    uint32_t nxt = w[i + 1];
    out[i] = __funnelshift_r(prev, nxt, sh);
    prev = nxt;
  }
}

// ----------------------------------------------------------------------------- mbarrier + bulk copy

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Barrier among the first `nthreads` threads of the block (whole warps), id 1..15.
__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for phase `parity` of an mbarrier.  Returns false (and raises
// NS_DEVERR_COPY_WAIT) if it did not complete within kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      raise_device_error(NS_DEVERR_COPY_WAIT);
      return false;
    }
  }
  return true;
}

// 1-D bulk async copy global -> shared (TMA engine, no tensor map, no multicast).
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// ----------------------------------------------------------------------------- staged byte ranges

// Copy global bytes [g0, g1) into shared memory at dst + (g - floor16(g0)),
// using the bulk-copy engine for the 16-byte-aligned part that lies inside the
// caller's buffer [buf0, buf1) and plain byte loads for what does not.
// The bulk part is issued by the calling thread (which must be a single
// thread) and signals `bar`; the function returns the number of bytes the
// barrier must expect (already armed via arrive.expect_tx).  The ragged bytes
// are NOT copied here: see copy_ragged().
struct Span {
  const uint8_t* g0;   // first wanted byte
  const uint8_t* g1;   // one past last wanted byte
};

__device__ __forceinline__ uintptr_t floor16(uintptr_t a) { return a & ~uintptr_t(15); }
__device__ __forceinline__ uintptr_t ceil16(uintptr_t a) { return (a + 15) & ~uintptr_t(15); }

// Bulk-copyable window of span s within the buffer [buf0, buf1).
__device__ __forceinline__ void bulk_window(Span s, const uint8_t* buf0, const uint8_t* buf1,
                                            uintptr_t* lo, uintptr_t* hi) {
  uintptr_t a = reinterpret_cast<uintptr_t>(s.g0), b = reinterpret_cast<uintptr_t>(s.g1);
  uintptr_t l = floor16(a), h = ceil16(b);
  if (l < reinterpret_cast<uintptr_t>(buf0)) l = ceil16(a);
  if (h > reinterpret_cast<uintptr_t>(buf1)) h = floor16(b);
  if (h < l) h = l;
  *lo = l;
  *hi = h;
}

// Issue the bulk part of span s into dst (dst corresponds to floor16(g0)).
// Returns bytes issued.  Single thread.
__device__ __forceinline__ uint32_t issue_span(uint8_t* dst, Span s, const uint8_t* buf0, const uint8_t* buf1,
                                               uint64_t* bar) {
  uintptr_t lo, hi;
  bulk_window(s, buf0, buf1, &lo, &hi);
  if (hi <= lo) return 0;
  uintptr_t base = floor16(reinterpret_cast<uintptr_t>(s.g0));
  uint32_t bytes = (uint32_t)(hi - lo);
  bulk_g2s(dst + (lo - base), reinterpret_cast<const void*>(lo), bytes, bar);
  return bytes;
}

// Same as issue_span, as bulk copies of at most `piece` bytes (a multiple of 16), all completing
// on `bar`: several copies in flight instead of one long one.
__device__ __forceinline__ uint32_t issue_span_pieces(uint8_t* dst, Span s, const uint8_t* buf0, const uint8_t* buf1,
                                                      uint64_t* bar, uint32_t piece) {
  uintptr_t lo, hi;
  bulk_window(s, buf0, buf1, &lo, &hi);
  if (hi <= lo) return 0;
  uintptr_t base = floor16(reinterpret_cast<uintptr_t>(s.g0));
  for (uintptr_t p = lo; p < hi; p += piece) {
    const uint32_t n = (uint32_t)min((uintptr_t)piece, hi - p);
    bulk_g2s(dst + (p - base), reinterpret_cast<const void*>(p), n, bar);
  }
  return (uint32_t)(hi - lo);
}

// Copy the bytes of span s that issue_span left out (at most 15 at each end),
// with plain loads.  Called by a whole warp after the barrier completed.
__device__ __forceinline__ void copy_ragged(uint8_t* dst, Span s, const uint8_t* buf0, const uint8_t* buf1,
                                            int lane) {
  uintptr_t lo, hi;
  bulk_window(s, buf0, buf1, &lo, &hi);
  uintptr_t a = reinterpret_cast<uintptr_t>(s.g0), b = reinterpret_cast<uintptr_t>(s.g1);
  uintptr_t base = floor16(a);
  if (hi <= lo) {  // nothing bulk-copied: the warp copies the whole span
    for (uintptr_t g = a + lane; g < b; g += 32) dst[g - base] = *reinterpret_cast<const uint8_t*>(g);
    return;
  }
  // head [a, lo) and tail [hi, b): each shorter than 16 bytes
  if (lane < 16) {
    uintptr_t g = a + lane;
    if (g < lo) dst[g - base] = *reinterpret_cast<const uint8_t*>(g);
  } else {
    uintptr_t g = hi + (lane - 16);
    if (g < b) dst[g - base] = *reinterpret_cast<const uint8_t*>(g);
  }
}

__device__ __forceinline__ bool span_has_ragged(Span s, const uint8_t* buf0, const uint8_t* buf1) {
  uintptr_t lo, hi;
  bulk_window(s, buf0, buf1, &lo, &hi);
  return hi <= lo || lo > reinterpret_cast<uintptr_t>(s.g0) || hi < reinterpret_cast<uintptr_t>(s.g1);
}

// Shared bytes a span needs when placed at a 16-byte boundary.
__device__ __host__ __forceinline__ uint32_t span_smem_bytes(uint64_t nbytes) {
  return (uint32_t)(((nbytes + 15 + 15) / 16) * 16);
}

// Programmatic dependent launch: wait until the previous grid of the stream has completed and its
// memory is visible (a no-op when this grid was launched without the attribute); let the next grid's
// CTAs be scheduled once every CTA of this grid has signalled or exited.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// ----------------------------------------------------------------------------- L2 prefetch hints

__device__ __forceinline__ void prefetch_l2_bulk(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// CTA `cta` of `ncta` asks L2 for its equal share of every range of `pf` (one thread calls this).
// Shares start and end on 16-byte boundaries; pieces of at most 64 KB.
__device__ __forceinline__ void l2_prefetch_share(const ns_l2_prefetch_t& pf, int cta, int ncta) {
#pragma unroll 1
  for (int i = 0; i < NS_L2_PREFETCH_RANGES; ++i) {
    const uint64_t n = pf.bytes[i];
    if (!n || !pf.ptr[i]) continue;
    const uint64_t lo = (n * (uint64_t)cta / (uint64_t)ncta) & ~uint64_t(15);
    const uint64_t hi = cta + 1 == ncta ? (n & ~uint64_t(15)) : ((n * (uint64_t)(cta + 1) / (uint64_t)ncta) & ~uint64_t(15));
    const uint8_t* base = static_cast<const uint8_t*>(pf.ptr[i]);
    for (uint64_t o = lo; o < hi; o += 65536u)
      prefetch_l2_bulk(base + o, (uint32_t)(hi - o < 65536u ? hi - o : 65536u));
  }
}

// ----------------------------------------------------------------------------- warp utilities

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace ns
