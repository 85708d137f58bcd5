// ns_peer_allreduce: the expert-parallel combine (a sum over the ranks of one node) through peer
// memory, for the small per-layer vectors of decode.
//
// Under expert parallelism every rank computes its local experts' weighted partial of the layer
// output (the residual on one rank) and the layer output is the sum over ranks -- the combine of
// neurostream's _ffn_block / moe_ffn (neurostream/model/gpt_oss.py:139-177, neurostream/moe/
// router.py:183-219) split by expert.  Each rank stores every value straight into every rank's
// receive slots over NVLink as one 64-bit word (value, epoch) -- the value and its arrival flag in
// one single-copy-atomic store, the low-latency packing of NCCL's LL protocol, so no fence and no
// separate flag -- and each rank sums, in rank order, the words whose epoch says they are this call's:
//
//   thread of CTA c, rank q:  slots[r][parity][q][i] = (data[i], epoch)   for every rank r, i in slice c
//                             wait slots[q][parity][r][i].epoch == epoch  for every rank r (bounded)
//                             data[i] = sum over r in rank order of slots[q][parity][r][i].value
//
// Every rank sums the same values in the same order, so all ranks hold identical bits.  The epoch is
// a per-CTA counter kept in device memory (one increment per call, in lockstep on every rank because
// every rank makes the same calls), so the call can sit in a CUDA graph and be replayed.  Receive
// slots alternate by epoch parity: a rank can be at most one call ahead of a peer, because finishing
// a call needs every peer's words of that call.  Plain peer stores and loads only (no multicast
// objects).  The wait is bounded: after ~1 s it raises NS_DEVERR_GRID_WAIT and returns.

namespace ns {

constexpr int kPeerThreads = 256;

__device__ __forceinline__ void st_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kPeerThreads) peer_allreduce_kernel(const ns_peer_reduce_t p) {
  const int c = blockIdx.x, G = gridDim.x, tid = threadIdx.x;
  const int W = p.world, q = p.rank;
  const int64_t per = (p.n + G - 1) / G, i0 = min(p.n, (int64_t)c * per), i1 = min(p.n, i0 + per);
  __shared__ uint32_t s_epoch;
  // launched with programmatic dependent launch: data and the counters are read after the wait; the
  // next kernel may start after it (the library's chain invariant: trigger only after the own wait)
  griddep_wait();
  griddep_launch_dependents();
  if (tid == 0) s_epoch = p.ctr[c] + 1u;
  __syncthreads();
  const uint32_t epoch = s_epoch, par = epoch & 1u;
  // 1. this rank's values, tagged with the epoch, into every rank's receive slot (its own included)
  for (int64_t i = i0 + tid; i < i1; i += kPeerThreads) {
    const uint64_t w = ((uint64_t)epoch << 32) | __float_as_uint(p.data[i]);
    for (int r = 0; r < W; ++r) st_sys_u64(p.slots[r] + ((int64_t)par * W + q) * p.cap + i, w);
  }
  // 2. + 3. wait for every rank's word of each element, then the sum in rank order
  const uint64_t* mine = p.slots[q] + (int64_t)par * W * p.cap;
  const uint64_t t0 = globaltimer_ns();
  bool late = false;
  for (int64_t i = i0 + tid; i < i1; i += kPeerThreads) {
    float s = 0.f;
    for (int r = 0; r < W; ++r) {
      uint64_t w = ld_sys_u64(mine + (int64_t)r * p.cap + i);
      while ((uint32_t)(w >> 32) != epoch && !late) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          raise_device_error(NS_DEVERR_GRID_WAIT);
          late = true;
        }
        w = ld_sys_u64(mine + (int64_t)r * p.cap + i);
      }
      s = __fadd_rn(s, __uint_as_float((uint32_t)w));
    }
    p.data[i] = s;
  }
  __syncthreads();
  if (tid == 0) p.ctr[c] = epoch;
}

}  // namespace ns

extern "C" int ns_peer_allreduce(const ns_peer_reduce_t* p, ns_stream_t stream) {
  using namespace ns;
  if (!p || p->world < 1 || p->world > NS_MAX_PEERS || p->rank < 0 || p->rank >= p->world)
    return fail(NS_ERR_INVALID, "ns_peer_allreduce: bad world/rank");
  if (p->n < 0 || p->n > p->cap || !p->data || !p->ctr)
    return fail(NS_ERR_INVALID, "ns_peer_allreduce: n=%lld outside the slot capacity %lld", (long long)p->n,
                (long long)p->cap);
  for (int r = 0; r < p->world; ++r)
    if (!p->slots[r]) return fail(NS_ERR_INVALID, "ns_peer_allreduce: missing peer %d", r);
  if (p->n == 0) return NS_OK;
  const int grid = (int)std::min<int64_t>((p->n + 1023) / 1024, NS_PEER_MAX_CTAS);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kPeerThreads);
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  NS_CUDA_TRY(cudaLaunchKernelEx(&cfg, peer_allreduce_kernel, *p));
  return NS_OK;
}

extern "C" int ns_peer_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return ns::fail(NS_ERR_INVALID, "ns_peer_alloc: bad arguments");
  NS_CUDA_TRY(cudaMalloc(ptr, bytes));
  NS_CUDA_TRY(cudaMemset(*ptr, 0, bytes));
  return NS_OK;
}

extern "C" int ns_peer_free(void* ptr) {
  if (ptr) NS_CUDA_TRY(cudaFree(ptr));
  return NS_OK;
}

extern "C" int ns_ipc_handle(const void* ptr, uint8_t* handle) {
  if (!ptr || !handle) return ns::fail(NS_ERR_INVALID, "ns_ipc_handle: null argument");
  cudaIpcMemHandle_t h;
  NS_CUDA_TRY(cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)));
  memcpy(handle, &h, sizeof h);
  return NS_OK;
}

extern "C" int ns_ipc_open(const uint8_t* handle, void** ptr) {
  if (!ptr || !handle) return ns::fail(NS_ERR_INVALID, "ns_ipc_open: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof h);
  NS_CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return NS_OK;
}

extern "C" int ns_ipc_close(void* ptr) {
  if (ptr) NS_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
  return NS_OK;
}
