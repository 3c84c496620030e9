// SwiGLU activation of the fused gate/up projection.
//
// needle computes F.silu(gate_proj(x)) * up_proj(x) (needle/model/llama.py:37)
// as two torch kernels with a bf16 round trip in between.  Here the gate and
// up halves come from one fused GEMM output [T, 2*I] and one pass writes
// [T, I]: out = rnd(rnd(silu(g)) * u), silu(g) = g / (1 + exp(-g)) in fp32,
// with the same two rounding points as the two torch ops.
#pragma once
#include "nb_common.cuh"

namespace nb {

template <typename T, int VEC>
__global__ void __launch_bounds__(256)
    silu_mul_kernel(const T* __restrict__ in, int64_t in_stride, T* __restrict__ out,
                    int64_t out_stride, int inter, int64_t total_vec) {
  // programmatic launch, as rmsnorm_kernel
  griddep_wait();
  griddep_launch_dependents();
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= total_vec) return;
  const int vpr = inter / VEC;
  const int64_t t = gid / vpr;
  const int c = (int)(gid - t * vpr) * VEC;
  const T* g = in + t * in_stride + c;
  const T* u = g + inter;
  T gv[VEC], uv[VEC], ov[VEC];
  if constexpr (VEC * sizeof(T) == 16) {
    *reinterpret_cast<uint4*>(gv) = __ldg(reinterpret_cast<const uint4*>(g));
    *reinterpret_cast<uint4*>(uv) = __ldg(reinterpret_cast<const uint4*>(u));
  } else {
#pragma unroll
    for (int e = 0; e < VEC; ++e) { gv[e] = g[e]; uv[e] = u[e]; }
  }
#pragma unroll
  for (int e = 0; e < VEC; ++e) {
    const float x = Dt<T>::to_f(gv[e]);
    // silu in fp32 with the fast exponential and divide: a few fp32 ulps from
    // torch's x / (1 + exp(-x)), below the bf16/fp16 rounding that follows
    // (fp32 itself keeps the exact forms)
    float s;
    if constexpr (sizeof(T) == 2) s = Dt<T>::round(__fdividef(x, 1.0f + __expf(-x)));
    else s = x / (1.0f + expf(-x));
    ov[e] = Dt<T>::from_f(s * Dt<T>::to_f(uv[e]));
  }
  T* o = out + t * out_stride + c;
  if constexpr (VEC * sizeof(T) == 16) {
    *reinterpret_cast<uint4*>(o) = *reinterpret_cast<uint4*>(ov);
  } else {
#pragma unroll
    for (int e = 0; e < VEC; ++e) o[e] = ov[e];
  }
}

}  // namespace nb

namespace nbh {

template <typename T>
int launch_silu_mul(const void* in, int64_t is, void* out, int64_t os, int T_, int inter,
                    cudaStream_t st) {
  constexpr int V16 = 16 / sizeof(T);
  const bool vec = inter % V16 == 0 && is % V16 == 0 && os % V16 == 0 &&
                   (uintptr_t)in % 16 == 0 && (uintptr_t)out % 16 == 0;
  const int threads = 256;
  const int64_t total = (int64_t)T_ * (vec ? inter / V16 : inter);
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute attr[1];
  pdl_config(cfg, attr, dim3((unsigned)((total + threads - 1) / threads)), dim3(threads), 0, st);
  auto kern = vec ? nb::silu_mul_kernel<T, V16> : nb::silu_mul_kernel<T, 1>;
  const cudaError_t e =
      cudaLaunchKernelEx(&cfg, kern, (const T*)in, is, (T*)out, os, inter, total);
  if (e != cudaSuccess) return fail(NB_ERR_CUDA, "silu_mul launch: %s", cudaGetErrorString(e));
  return check_launch("silu_mul");
}

}  // namespace nbh

extern "C" {

int nb_silu_mul(const void* gate_up, int64_t gate_up_stride, void* out, int64_t out_stride,
                int num_tokens, int intermediate, int dtype, void* stream) {
  using namespace nbh;
  if (!valid_dtype(dtype)) return fail(NB_ERR_INVALID_ARG, "invalid dtype %d", dtype);
  if (!gate_up || !out) return fail(NB_ERR_INVALID_ARG, "null pointer");
  if (num_tokens < 0 || intermediate <= 0) return fail(NB_ERR_INVALID_ARG, "bad sizes");
  if (gate_up_stride < 2ll * intermediate || out_stride < intermediate)
    return fail(NB_ERR_INVALID_ARG, "row stride too small");
  if (num_tokens == 0) return NB_OK;
  cudaStream_t st = (cudaStream_t)stream;
  switch (dtype) {
    case NB_DTYPE_F32: return launch_silu_mul<float>(gate_up, gate_up_stride, out, out_stride, num_tokens, intermediate, st);
    case NB_DTYPE_F16: return launch_silu_mul<__half>(gate_up, gate_up_stride, out, out_stride, num_tokens, intermediate, st);
    default: return launch_silu_mul<__nv_bfloat16>(gate_up, gate_up_stride, out, out_stride, num_tokens, intermediate, st);
  }
}

}  // extern "C"
