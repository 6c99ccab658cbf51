// m4-b200.cuh -- the ggml-cuda side of the M4 ops on B200: the three launchers ggml-cuda's
// compute_forward dispatches GGML_OP_M4_{WKB,KQKV,PHASE} to (ggml-cuda.cu:2504-2512 in the
// reference's patched tree; they replace patches/ggml-m4/m4-{wkb,kqkv,phase}.cu and keep their
// names and signatures) and the supports_op check for the three ops (ggml-cuda.cu:5848-5885).
// Each launcher is a thin shim over the C ABI of libm4b (include/m4b.h).
#pragma once

#include "common.cuh"

void ggml_cuda_m4_wkb(ggml_backend_cuda_context & ctx, ggml_tensor * dst);
void ggml_cuda_m4_kqkv(ggml_backend_cuda_context & ctx, ggml_tensor * dst);
void ggml_cuda_m4_phase(ggml_backend_cuda_context & ctx, ggml_tensor * dst);

// true when libm4b supports the node's shapes and types (no CUDA call; tensors need no memory yet)
bool ggml_cuda_m4_supports_op(const ggml_tensor * op);
