/*
 * ns_b200.h -- C ABI of the B200 (sm_100a) decode hot path of neurostream.
 *
 * The reference (hareramray/nurostream, package `neurostream`) is pure Python;
 * its hot path is Python/Triton with no FFI.  Each entry point below replaces
 * one Python operator of that path and keeps its argument meaning; the cited
 * reference lines are the operator it stands in for.  The Python side binds
 * this header with ctypes (nurostream_b200/_lib.py) and mirrors the reference's
 * operator names on top of it.
 *
 * Conventions
 *  - All buffers are caller-owned device memory passed as raw pointers plus
 *    sizes; the library never allocates or frees caller memory.
 *  - Every call is asynchronous and ordered on `stream`; none synchronises the
 *    host except ns_device_error().
 *  - Return value: NS_OK (0) or a negative ns_status; ns_last_error() returns a
 *    message for the last failure on the calling host thread.
 *  - Device-side waits are bounded (about one second); a wait that runs out
 *    sets a bit in the per-device error word read by ns_device_error().
 */
#ifndef NS_B200_H
#define NS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NS_ABI_VERSION 2
#define NS_MAX_TOKENS 8     /* tokens per fused GEMV or MoE-decode call */
#define NS_MAX_TOPK 16      /* experts used per token */
#define NS_MAX_EXPERTS 512  /* experts in one stacked tensor */

typedef struct CUstream_st* ns_stream_t; /* identical to cudaStream_t */

/* GGUF tensor type ids (on-disk values, neurostream/format/gguf.py:19-35). */
enum ns_ggml_type {
  NS_GGML_F32 = 0,
  NS_GGML_F16 = 1,
  NS_GGML_Q4_0 = 2,
  NS_GGML_Q8_0 = 8,
  NS_GGML_Q4_K = 12,
  NS_GGML_Q5_K = 13,
  NS_GGML_Q6_K = 14,
  NS_GGML_BF16 = 30,
  NS_GGML_MXFP4 = 39
};

/* Element types of activations and outputs. */
enum ns_float_type { NS_F32 = 0, NS_F16 = 1, NS_BF16 = 2 };

enum ns_status {
  NS_OK = 0,
  NS_ERR_INVALID = -1,     /* null pointer, bad count or stride */
  NS_ERR_UNSUPPORTED = -2, /* type or shape outside what the kernels handle */
  NS_ERR_SIZE = -3,        /* buffer smaller than the shape requires */
  NS_ERR_CUDA = -4,        /* a CUDA runtime call failed */
  NS_ERR_TIMEOUT = -5      /* a bounded device wait ran out */
};

/* Router variants. */
enum ns_route_mode {
  NS_ROUTE_TOPK_SOFTMAX = 0,     /* GPT-OSS: top-k of biased logits, softmax over the k
                                    (neurostream/model/gpt_oss.py:116-121) */
  NS_ROUTE_SOFTMAX_TOPK_NORM = 1 /* Qwen3-MoE: softmax, top-k, renormalise
                                    (neurostream/moe/router.py:59-69) */
};

/* Expert activations. */
enum ns_act_mode {
  NS_ACT_CLAMPED_SWIGLU = 0, /* GPT-OSS (neurostream/model/gpt_oss.py:61-70) */
  NS_ACT_SILU_MUL = 1        /* Qwen3 silu(gate)*up (neurostream/moe/router.py:208) */
};

/* Bits of the per-device error word. */
#define NS_DEVERR_GRID_WAIT 1u  /* grid-wide barrier ran out */
#define NS_DEVERR_COPY_WAIT 2u  /* bulk-copy completion wait ran out */
#define NS_DEVERR_ROUTE 4u      /* an invalid expert id, token id or position */

const char* ns_last_error(void);
int ns_abi_version(void);

/* Block layout of a GGML type: elements and bytes per block
 * (neurostream/format/gguf.py:39-55). */
int ns_type_layout(int ggml_type, int* block_elems, int* block_bytes);

/* Read (and optionally clear) the error word of the current device.
 * Synchronises the device. */
int ns_device_error(uint32_t* bits, int clear);

/*
 * Expand GGML bytes to floats, bit-exact with the reference.
 * Replaces neurostream/compute/quant.py:153-184 `dequantize(raw, dtype, n_elements, out_dtype)`.
 * raw: raw_bytes bytes of type ggml_type; out: n_elements values of out_dtype.
 * Decodes whole blocks and truncates to n_elements, like the reference.
 */
int ns_dequant(const uint8_t* raw, size_t raw_bytes, int ggml_type, int64_t n_elements,
               void* out, int out_dtype, ns_stream_t stream);

/*
 * Fused dequant-GEMV straight from GGUF bytes: y[t, n] = sum_k x[t, k] * W[n, k],
 * fp32 accumulation, for T <= NS_MAX_TOKENS activation rows.
 * Replaces neurostream/compute/triton_kernels.py:199-228 `fused_gemv(raw, dtype, x, n_rows, K, out_dtype)`
 * (kernels :37-174).  w: n_rows rows of row_bytes(ggml_type, K) bytes (w_bytes >= that);
 * x: T rows of K values of x_dtype, row stride x_stride elements;
 * y: T rows of n_rows values of y_dtype, row stride y_stride elements.
 * Types: MXFP4, Q8_0, Q4_K, Q6_K.
 */
int ns_gemv(const uint8_t* w, size_t w_bytes, int ggml_type, int n_rows, int K,
            const void* x, int x_dtype, int64_t x_stride, int T,
            void* y, int y_dtype, int64_t y_stride, ns_stream_t stream);

/*
 * MoE router on device: logits = h @ W^T (+ b), then top-k and softmax per `mode`.
 * Replaces neurostream/model/gpt_oss.py:116-121 `GptOssModel._route` and
 * neurostream/moe/router.py:59-69 `route` (without their host sync).
 * h: T x H (h_dtype), W: E x H (w_dtype, one of NS_F32/NS_F16/NS_BF16), b: E fp32 or NULL.
 * ids: T x k int32 (descending score), weights: T x k fp32, logits: T x E fp32 or NULL.
 */
int ns_moe_route(const void* h, int h_dtype, int T, int H,
                 const void* w, int w_dtype, const float* b, int E, int k, int mode,
                 int32_t* ids, float* weights, float* logits, ns_stream_t stream);

/*
 * One fused MoE decode layer: RMSNorm -> router -> top-k -> for every routed
 * expert gate/up (+bias) -> activation -> down (+bias) -> weighted combine
 * (+ residual), as ONE launch of one CTA per SM, every CTA resident at once
 * (a cooperative launch for the CUDA-core kernel; the tensor-core kernel's
 * plain launch relies on one CTA filling an SM, its grid-wide waits bounded).
 * Replaces neurostream/model/gpt_oss.py:123-177 `GptOssModel._ffn_block` (with
 * stream_expert_ffn, neurostream/compute/blockffn.py:396-449) and
 * neurostream/moe/router.py:173-219 `moe_ffn`.
 *
 * Expert parallelism: the stacked expert tensors hold only experts
 * [expert_lo, expert_hi) (local expert i is global expert expert_lo + i).
 * Routing is computed over all n_expert; only local experts contribute, so
 * summing `out` over ranks (with residual added on one rank only) gives the
 * full layer.
 */
/*
 * Byte ranges a kernel asks L2 to fetch while it runs (cp.async.bulk.prefetch.L2,
 * a hint: nothing waits for it, nothing is written).  Meant for the weights of
 * the kernels that follow in the stream, so that HBM works while this kernel is
 * latency-bound (routing, split merges) and they find their weights in L2.  Each
 * CTA prefetches an equal share.  Ranges start on 16 bytes; unused slots have
 * bytes = 0.  No reference counterpart (the reference has no device pipeline).
 */
#define NS_L2_PREFETCH_RANGES 4
typedef struct ns_l2_prefetch {
  const void* ptr[NS_L2_PREFETCH_RANGES];
  uint64_t bytes[NS_L2_PREFETCH_RANGES];
} ns_l2_prefetch_t;

typedef struct ns_moe_layer {
  int T;            /* tokens, 1..NS_MAX_TOKENS */
  int H;            /* hidden size (n_embd) */
  int F;            /* expert ffn width */
  int n_expert;     /* experts seen by the router */
  int expert_lo;    /* first expert held by these tensors */
  int expert_hi;    /* one past the last */
  int k;            /* experts per token */
  int route_mode;   /* ns_route_mode */
  int act_mode;     /* ns_act_mode */
  int ggml_type;    /* type of gate/up/down expert tensors */
  float alpha;      /* clamped-SwiGLU sigmoid slope (1.702) */
  float limit;      /* clamped-SwiGLU clamp (7.0) */
  float rms_eps;    /* RMSNorm epsilon, used when norm_w != NULL */
  int add_residual; /* 1: out = x + moe, 0: out = moe */
  const float* x;   /* T x H fp32 layer input (residual stream) */
  const float* norm_w;  /* H fp32 RMSNorm weight, or NULL for h = x */
  const void* router_w; /* n_expert x H */
  int router_dtype;     /* NS_F32 / NS_F16 / NS_BF16 */
  const float* router_b;  /* n_expert fp32 or NULL */
  const uint8_t* gate_w;  /* local experts x F rows of row_bytes(type, H) */
  const uint8_t* up_w;    /* same layout as gate_w */
  const uint8_t* down_w;  /* local experts x H rows of row_bytes(type, F) */
  const float* gate_b;    /* local experts x F fp32, or NULL */
  const float* up_b;      /* local experts x F fp32, or NULL */
  const float* down_b;    /* local experts x H fp32, or NULL */
  float* out;             /* T x H fp32 */
  int32_t* ids;           /* T x k int32 routed experts, or NULL */
  float* weights;         /* T x k fp32 routing weights, or NULL */
  ns_l2_prefetch_t l2;    /* L2 prefetch hint (zeros: none) */
} ns_moe_layer_t;

/* Workspace bytes a layer call with 1..p->T tokens needs (zeroed once with
 * ns_moe_workspace_init; one workspace serves any number of stream-ordered
 * calls on one device).
 * The tensor-core layer kernel is launched with programmatic dependent launch:
 * it may read norm_w and router_w before the previous kernel on the stream has
 * finished, if that kernel signals its dependents early (the layer kernel
 * itself does so). Do not write a layer's weights in such a kernel; x, the
 * workspace and everything else are read only after the previous kernel
 * completes. */
int ns_moe_workspace_bytes(const ns_moe_layer_t* p, size_t* bytes);
int ns_moe_workspace_init(void* workspace, size_t bytes, ns_stream_t stream);
int ns_moe_decode_layer(const ns_moe_layer_t* p, void* workspace, size_t workspace_bytes,
                        ns_stream_t stream);

/*
 * ns_moe_decode_layer without a caller workspace and without any allocation.
 * No counterpart in the reference (its Python layer allocates torch tensors
 * per call); it exists for callers that cannot allocate device memory per
 * call: a plain C / FFI host binding only this header, with no caching
 * allocator, or a decoder whose weight cache has budgeted all free HBM --
 * cudaMalloc/cudaFree there would synchronise the device mid-step and
 * fragment that budget.
 *
 * Same computation and results as ns_moe_decode_layer; the scratch comes from
 * one fixed array of NS_MOE_STATIC_SCRATCH_BYTES linked into the library, one
 * per device.  A call whose own scratch -- what the kernel chosen for this
 * call's T needs, which can be less than ns_moe_workspace_bytes reports for a
 * layer sized for up to T tokens -- exceeds that returns NS_ERR_SIZE without
 * launching (T=1, k=4, H=F=2880, 128 experts needs 349,696).
 * The first call on a device (that device current) resolves the array's
 * address and clears its first 1 KiB (the grid-barrier word) with a
 * synchronous memset: make it before any stream capture.  Every launch clears
 * its own counters, so nothing else needs to start at zero.  The address is
 * cached per device ordinal: cudaDeviceReset after the first call is not
 * supported.
 * Calls that overlap on the GPU (unordered streams) race on the one array and
 * give wrong results; calls ordered on one stream are safe.
 */
#define NS_MOE_STATIC_SCRATCH_BYTES (1024 * 1024)
int ns_moe_decode_layer_static(const ns_moe_layer_t* p, ns_stream_t stream);

/*
 * MoE prefill of T tokens (1..65536) as a grouped expert GEMM on the tcgen05
 * tensor cores: RMSNorm -> router -> top-k -> tokens grouped by expert (<= 16
 * per group) -> gate/up (+bias) -> activation -> down (+bias) -> weighted
 * combine in ascending expert order (+ residual).  Same parameters, results
 * (to fp32 rounding) and expert-parallel contract as ns_moe_decode_layer, for
 * any T; every expert's weights stream from HBM once per group of its tokens.
 * Replaces the prefill walk of neurostream/compute/blockffn.py:171-176, 220-229
 * (per-expert dequantize + matmul over blocks) and neurostream/moe/router.py:
 * 158-166.  MXFP4 experts only (NS_ERR_UNSUPPORTED otherwise); H and F
 * multiples of 64 up to 8192; expert tensors, router_w, x and out 16-byte
 * aligned.
 * Workspace: ns_moe_prefill_workspace_bytes, 256-byte aligned, no
 * initialisation needed.  Six stream-ordered launches, no host synchronisation.
 */
int ns_moe_prefill_workspace_bytes(const ns_moe_layer_t* p, size_t* bytes);
int ns_moe_prefill_grouped(const ns_moe_layer_t* p, void* workspace, size_t workspace_bytes,
                           ns_stream_t stream);

/*
 * Dense projection with bf16 weights, fp32 activations and fp32 accumulation
 * (batch 1): for each segment s, y_s = residual_s + (W_s @ x' + bias_s), where
 * x' = rms_norm(x, norm_w) (x * rsqrt(mean(x^2) + eps) * norm_w) when norm_w is
 * given, else x.  Up to NS_DENSE_MAX_SEG matrices with the same K run as one
 * launch over their concatenated rows (q, k and v of an attention block).
 * Replaces neurostream/model/qwen3.py:169-194 `Qwen3Model._linear` on float
 * weights (`x @ W.T`) and neurostream/model/gpt_oss.py:97-99 `_biased_linear`,
 * with neurostream/compute/ops.py:14-20 `rms_norm` before it and the residual
 * add of gpt_oss.py:101-114 after it.
 * K a multiple of 8 up to 8192; w, x, norm_w 16-byte aligned.
 */
#define NS_DENSE_MAX_SEG 4
typedef struct ns_dense_seg {
  const void* w;          /* rows x K weights (w_dtype), row-major */
  int rows;
  const float* bias;      /* rows fp32, or NULL */
  const float* residual;  /* rows fp32, or NULL */
  float* y;               /* rows fp32 */
} ns_dense_seg_t;

typedef struct ns_dense_gemv {
  int K;
  int w_dtype;            /* NS_BF16 */
  int n_seg;              /* 1..NS_DENSE_MAX_SEG */
  ns_dense_seg_t seg[NS_DENSE_MAX_SEG];
  const float* x;         /* K fp32 */
  const float* norm_w;    /* K fp32 RMSNorm weight, or NULL */
  float rms_eps;
  ns_l2_prefetch_t l2;    /* L2 prefetch hint (zeros: none) */
} ns_dense_gemv_t;

int ns_dense_gemv(const ns_dense_gemv_t* p, ns_stream_t stream);

/*
 * One decode token of attention with sinks over an fp32 KV cache.
 * Replaces the core of neurostream/model/gpt_oss.py:101-114
 * `GptOssModel._attention_block`: apply_rope on q and the new key
 * (neurostream/compute/ops.py:136-151), KVCache.append
 * (neurostream/model/qwen3.py:74-85), repeat_kv (ops.py:154-159) and
 * sink_attention (gpt_oss.py:73-87), with its sliding window.
 * qkv: the un-rotated projection output, q (n_head*head_dim) then k then v
 * (n_head_kv*head_dim each).  The token's position is read from device memory
 * (*pos), so one captured graph serves every position; its key and value are
 * written to cache slot *pos.  Keys kp with (window ? pos - window < kp : 0 <= kp)
 * and kp <= pos are visible.  head_dim 64; at most 8 query heads per kv head.
 */
typedef struct ns_attn_decode {
  int n_head;
  int n_head_kv;
  int head_dim;
  int max_ctx;              /* positions each cache holds */
  int window;               /* 0: full causal attention; > 0: sliding window */
  float scale;              /* 1 / sqrt(head_dim) */
  const int32_t* pos;       /* device int32: position of the token */
  const float* qkv;         /* fp32 projection output (see above) */
  const float* rope_cos;    /* max_ctx x head_dim fp32 (the model's RoPE / YaRN tables) */
  const float* rope_sin;
  const float* sinks;       /* n_head fp32 sink logits, or NULL */
  float* k_cache;           /* n_head_kv x max_ctx x head_dim fp32 */
  float* v_cache;
  float* out;               /* n_head*head_dim fp32 */
  ns_l2_prefetch_t l2;      /* L2 prefetch hint (zeros: none) */
} ns_attn_decode_t;

/* Workspace of ns_attn_decode: currently 0 bytes (the key splits of a kv head
 * form one thread-block cluster and merge through distributed shared memory);
 * the argument is kept so that a later version may ask for one. */
int ns_attn_workspace_bytes(const ns_attn_decode_t* p, size_t* bytes);
int ns_attn_decode(const ns_attn_decode_t* p, void* workspace, size_t workspace_bytes, ns_stream_t stream);

/*
 * A whole attention block for one decode token as ONE cooperative launch:
 * out = x + W_o attn(rope(q), rope(k), v) + b_o with q, k, v = W_{q,k,v}
 * rms_norm(x, norm_w) + b -- ns_dense_gemv (q/k/v), ns_attn_decode and
 * ns_dense_gemv (o-proj) without the kernel boundaries; one ring of
 * shared-memory stages per SM streams its q/k/v rows, its share of the key /
 * value history and its o-proj rows back to back.
 * Replaces neurostream/model/gpt_oss.py:101-114 `GptOssModel._attention_block`
 * (with rms_norm, _biased_linear, apply_rope, KVCache.append, repeat_kv and
 * sink_attention).  head_dim 64; at most 8 query heads per kv head; H and
 * n_head*64 at most 4096 columns.  The workspace (ns_attn_block_workspace_bytes,
 * 256-byte aligned) is zeroed once; calls ordered on one stream may share it.
 */
typedef struct ns_attn_block {
  int H;                    /* hidden size */
  int n_head;
  int n_head_kv;
  int head_dim;
  int max_ctx;              /* positions each cache holds */
  int window;               /* 0: full causal attention; > 0: sliding window */
  float rms_eps;
  float scale;              /* 1 / sqrt(head_dim) */
  const float* x;           /* H fp32 residual stream */
  const float* norm_w;      /* H fp32 (attn_norm) */
  const void* wq;           /* n_head*head_dim x H bf16 */
  const void* wk;           /* n_head_kv*head_dim x H bf16 */
  const void* wv;           /* n_head_kv*head_dim x H bf16 */
  const float* bq;          /* fp32 biases, or NULL */
  const float* bk;
  const float* bv;
  const void* wo;           /* H x n_head*head_dim bf16 */
  const float* bo;          /* H fp32, or NULL */
  const float* sinks;       /* n_head fp32 sink logits, or NULL */
  const int32_t* pos;       /* device int32: position of the token */
  const float* rope_cos;    /* max_ctx x head_dim fp32 */
  const float* rope_sin;
  float* k_cache;           /* n_head_kv x max_ctx x head_dim fp32 */
  float* v_cache;
  float* out;               /* H fp32 */
} ns_attn_block_t;

int ns_attn_block_workspace_bytes(const ns_attn_block_t* p, size_t* bytes);
int ns_attn_block(const ns_attn_block_t* p, void* workspace, size_t workspace_bytes, ns_stream_t stream);

/*
 * The embedding row of the token *token (device int32) widened to fp32:
 * neurostream/model/qwen3.py:266-275 `Qwen3Model.embed` (`W[tokens]`).
 * table: rows x H of dtype (NS_F32 / NS_F16 / NS_BF16).
 */
int ns_embed(const void* table, int dtype, int64_t rows, int H, const int32_t* token, float* out,
             ns_stream_t stream);

/*
 * Sum of n fp32 values over the `world` ranks of one node (one process per
 * GPU), in place in `data`, through peer memory: the expert-parallel combine
 * that follows each MoE layer (every rank holds its local experts' partial of
 * the layer output; neurostream/model/gpt_oss.py:139-177 and
 * neurostream/moe/router.py:183-219 sum the experts' contributions).  Every
 * rank stores each value into every rank's receive slots as one 64-bit word
 * (value, call epoch) over NVLink, and sums, in rank order, the words of this
 * call that arrived in its own memory; all ranks end with identical bits.  No
 * reference counterpart for the transport (the reference runs on one device).
 *
 * slots[r]: rank r's receive area, 2 * world * cap uint64 words, allocated by
 * its owner with ns_peer_alloc (zeroed) and mapped on the other ranks with
 * ns_ipc_handle / ns_ipc_open.  ctr: this rank's NS_PEER_MAX_CTAS uint32 call
 * counters (zeroed).  Every rank must make the same sequence of calls with the
 * same n.  The wait for the peers is bounded (~1 s); one that runs out raises
 * NS_DEVERR_GRID_WAIT.  Stream-ordered, graph-capturable, launched with
 * programmatic dependent launch.
 */
#define NS_MAX_PEERS 8
#define NS_PEER_MAX_CTAS 32
typedef struct ns_peer_reduce {
  int world, rank;
  int64_t n;                     /* floats to sum, <= cap */
  int64_t cap;                   /* words per receive slot */
  float* data;                   /* n fp32, this rank's input and the sum */
  uint64_t* slots[NS_MAX_PEERS]; /* rank r's receive area (mapped) */
  uint32_t* ctr;                 /* this rank's call counters */
} ns_peer_reduce_t;
int ns_peer_allreduce(const ns_peer_reduce_t* p, ns_stream_t stream);
int ns_peer_alloc(size_t bytes, void** ptr);
int ns_peer_free(void* ptr);
int ns_ipc_handle(const void* ptr, uint8_t* handle);      /* 64-byte cudaIpcMemHandle_t */
int ns_ipc_open(const uint8_t* handle, void** ptr);
int ns_ipc_close(void* ptr);

/*
 * Kernel choice of ns_moe_decode_layer (diagnostic and benchmarking aid; no
 * reference counterpart).  0 (default): the tcgen05 tensor-core kernel for
 * layers it takes (MXFP4 experts, T <= 2, H and F multiples of 64, 16-byte
 * aligned expert tensors), the CUDA-core / mma.sync kernel otherwise; 1: always
 * the latter; 2: the tensor-core kernel or NS_ERR_UNSUPPORTED.  Process-wide.
 */
int ns_moe_select_kernel(int path);

/*
 * Phase tracer of the fused layer (profiling aid; no reference counterpart --
 * the reference times with time.perf_counter around whole calls).  While set,
 * every ns_moe_decode_layer and ns_attn_block launch on the current device
 * writes, per CTA,
 * NS_TRACE_EVENTS globaltimer stamps (ns) to buf[cta * NS_TRACE_EVENTS + event].
 * ns_moe_prefill_grouped's two GEMM launches write per CTA their start and end
 * stamps (ns) and each role's SM clock cycles spent waiting (producer,
 * repack, MMA, epilogue), the gate/up launch at buf and the down launch at
 * buf + grid * NS_TRACE_EVENTS when buf holds twice the minimum (else at buf).
 * buf = NULL switches tracing off.  buf must hold grid * NS_TRACE_EVENTS uint64.
 */
#define NS_TRACE_EVENTS 16
int ns_moe_set_trace(uint64_t* buf, size_t bytes);

/*
 * Synthetic tensors for benchmarks and tests (no reference counterpart: the
 * reference's configurations are synthetic inputs).  Fills `count` bytes
 * (quantized `kind` = ggml type) or `count` values (kind = NS_SYNTH_F32/BF16)
 * starting at element/byte `start` of the stream (seed, stream); the host twin
 * is nurostream_b200/synth.py and agrees bit for bit.
 */
#define NS_SYNTH_F32 1000
#define NS_SYNTH_BF16 1001
int ns_synth_fill(void* dst, uint64_t count, int kind, uint64_t seed, uint64_t stream,
                  uint64_t start, float sigma, int e_lo, int e_hi, float scale_mult,
                  ns_stream_t s);

#ifdef __cplusplus
}
#endif
#endif /* NS_B200_H */
