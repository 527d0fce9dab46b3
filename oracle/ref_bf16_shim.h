/*
 * ref_bf16_shim.h — TEST INFRASTRUCTURE ONLY. Pre-include (nvcc -include) that
 * builds the reference's unmodified src/kernels.cu as a bfloat16 instance: the CUDA
 * fp16/bf16/cuBLAS headers are pulled in first under their own names, then the
 * reference's `half` type and its two conversion calls are renamed to their
 * bfloat16 counterparts. Used only by oracle/Makefile for oracle/_ref/.
 */
#pragma once
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cublas_v2.h>
#define half __nv_bfloat16
#define __half2float __bfloat162float
#define __float2half __float2bfloat16
