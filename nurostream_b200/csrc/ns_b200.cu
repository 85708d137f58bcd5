// Single translation unit of libns_b200.so: the kernels share the per-device
// error word (abi.cu), so they are compiled together rather than with
// relocatable device code.
#include "abi.cu"
#include "dequant.cu"
#include "dense.cu"
#include "attn.cu"
#include "gemv.cu"
#include "moe.cu"
#include "prefill.cu"
#include "attn_block.cu"
#include "synth.cu"
#include "peer.cu"
