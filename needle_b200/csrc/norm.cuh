// RMSNorm and residual-add + RMSNorm.
//
// One CTA per token row.  Pass 1 forms h (= x, or residual + x rounded to the
// storage type), writes residual_out, and accumulates sum(h^2) in fp32;
// pass 2 normalises.  Each thread revisits exactly the elements it produced
// in pass 1, so in-place use (out == x, residual_out == residual) is safe.
// Rounding points follow needle/layers/norm.py:14-17:
//   var = mean(float(h)^2);  r = 1 / sqrt(var + eps)
//   y   = rnd(w * rnd(float(h) * r))
// The fp32 sum runs in a different order than torch's CPU reduction, so r
// can differ from the reference in its last bit.
#pragma once
#include "nb_common.cuh"

namespace nb {

template <typename T, int VEC, bool ADD>
__global__ void __launch_bounds__(1024)
    rmsnorm_kernel(const T* x, int64_t xs, const T* res, int64_t rs, const T* __restrict__ w,
                   T* out, int64_t os, T* res_out, int64_t ros, int hidden, float eps) {
  // launched with programmatic stream serialisation: the launch overlaps the
  // previous kernel's tail; every read waits for that kernel's results
  griddep_wait();
  griddep_launch_dependents();
  __shared__ float red[32];
  const int row = blockIdx.x;
  const T* xr = x + (int64_t)row * xs;
  const T* rr = ADD ? res + (int64_t)row * rs : nullptr;
  T* hr = ADD ? res_out + (int64_t)row * ros : nullptr;
  T* orow = out + (int64_t)row * os;
  const int nvec = hidden / VEC;
  if (VEC * sizeof(T) == 16 && nvec <= (int)blockDim.x) {
    // One vector per thread (every decode shape up to hidden 8192): the row
    // stays in registers between the two passes and the weight load is
    // issued with the first loads, so the kernel makes one memory round trip.
    const int i = threadIdx.x;
    const bool mine = i < nvec;
    T hv[VEC], wv[VEC];
    float ss = 0.f;
    if (mine) {
      *reinterpret_cast<uint4*>(hv) = *reinterpret_cast<const uint4*>(xr + i * VEC);
      *reinterpret_cast<uint4*>(wv) = __ldg(reinterpret_cast<const uint4*>(w + i * VEC));
      if constexpr (ADD) {
        T rv[VEC];
        *reinterpret_cast<uint4*>(rv) = *reinterpret_cast<const uint4*>(rr + i * VEC);
#pragma unroll
        for (int e = 0; e < VEC; ++e)
          hv[e] = Dt<T>::from_f(__fadd_rn(Dt<T>::to_f(rv[e]), Dt<T>::to_f(hv[e])));
        *reinterpret_cast<uint4*>(hr + i * VEC) = *reinterpret_cast<uint4*>(hv);
      }
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const float f = Dt<T>::to_f(hv[e]);
        ss = __fadd_rn(ss, __fmul_rn(f, f));
      }
    }
    ss = warp_sum(ss);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (warp == 0) {
      float v = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
      v = warp_sum(v);
      if (lane == 0) red[0] = v;
    }
    __syncthreads();
    if (mine) {
      const float var = __fdiv_rn(red[0], (float)hidden);
      const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const float xn = Dt<T>::round(__fmul_rn(Dt<T>::to_f(hv[e]), r));
        hv[e] = Dt<T>::from_f(__fmul_rn(Dt<T>::to_f(wv[e]), xn));
      }
      *reinterpret_cast<uint4*>(orow + i * VEC) = *reinterpret_cast<uint4*>(hv);
    }
    return;
  }
  float ss = 0.f;
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    T hv[VEC];
    if constexpr (VEC * sizeof(T) == 16) {
      *reinterpret_cast<uint4*>(hv) = *reinterpret_cast<const uint4*>(xr + i * VEC);
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) hv[e] = xr[i * VEC + e];
    }
    if constexpr (ADD) {
      T rv[VEC];
      if constexpr (VEC * sizeof(T) == 16) {
        *reinterpret_cast<uint4*>(rv) = *reinterpret_cast<const uint4*>(rr + i * VEC);
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) rv[e] = rr[i * VEC + e];
      }
#pragma unroll
      for (int e = 0; e < VEC; ++e)
        hv[e] = Dt<T>::from_f(__fadd_rn(Dt<T>::to_f(rv[e]), Dt<T>::to_f(hv[e])));
      if constexpr (VEC * sizeof(T) == 16) {
        *reinterpret_cast<uint4*>(hr + i * VEC) = *reinterpret_cast<uint4*>(hv);
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) hr[i * VEC + e] = hv[e];
      }
    }
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const float f = Dt<T>::to_f(hv[e]);
      ss = __fadd_rn(ss, __fmul_rn(f, f));
    }
  }
  ss = warp_sum(ss);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  if (warp == 0) {
    float v = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
    v = warp_sum(v);
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  const float var = __fdiv_rn(red[0], (float)hidden);
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
  const T* src = ADD ? hr : xr;
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    T hv[VEC], wv[VEC];
    if constexpr (VEC * sizeof(T) == 16) {
      *reinterpret_cast<uint4*>(hv) = *reinterpret_cast<const uint4*>(src + i * VEC);
      *reinterpret_cast<uint4*>(wv) = __ldg(reinterpret_cast<const uint4*>(w + i * VEC));
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) { hv[e] = src[i * VEC + e]; wv[e] = w[i * VEC + e]; }
    }
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const float xn = Dt<T>::round(__fmul_rn(Dt<T>::to_f(hv[e]), r));
      hv[e] = Dt<T>::from_f(__fmul_rn(Dt<T>::to_f(wv[e]), xn));
    }
    if constexpr (VEC * sizeof(T) == 16) {
      *reinterpret_cast<uint4*>(orow + i * VEC) = *reinterpret_cast<uint4*>(hv);
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) orow[i * VEC + e] = hv[e];
    }
  }
}

}  // namespace nb

namespace nbh {

template <typename T, bool ADD>
int launch_norm(const void* x, int64_t xs, const void* res, int64_t rs, const void* w, void* out,
                int64_t os, void* ro, int64_t ros, int T_, int hidden, float eps,
                cudaStream_t st) {
  constexpr int V16 = 16 / sizeof(T);
  const bool vec_ok = hidden % V16 == 0 && xs % V16 == 0 && os % V16 == 0 &&
                      (!ADD || (rs % V16 == 0 && ros % V16 == 0)) && (uintptr_t)x % 16 == 0 &&
                      (uintptr_t)w % 16 == 0 && (uintptr_t)out % 16 == 0 &&
                      (!ADD || ((uintptr_t)res % 16 == 0 && (uintptr_t)ro % 16 == 0));
  // One CTA per row and (up to 1024) one vector per thread, so each thread's
  // chain of loads is short: the kernel is latency-bound at decode batch sizes.
  const int nvec = vec_ok ? hidden / V16 : hidden;
  int threads = 32;
  while (threads < 1024 && threads < nvec) threads *= 2;
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute attr[1];
  pdl_config(cfg, attr, dim3(T_), dim3(threads), 0, st);
  auto kern = vec_ok ? nb::rmsnorm_kernel<T, V16, ADD> : nb::rmsnorm_kernel<T, 1, ADD>;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, (const T*)x, xs, (const T*)res, rs,
                                           (const T*)w, (T*)out, os, (T*)ro, ros, hidden, eps);
  if (e != cudaSuccess) return fail(NB_ERR_CUDA, "rmsnorm launch: %s", cudaGetErrorString(e));
  return check_launch(ADD ? "fused_add_rmsnorm" : "rmsnorm");
}

template <bool ADD>
int norm_entry(const void* x, int64_t xs, const void* res, int64_t rs, const void* w, void* out,
               int64_t os, void* ro, int64_t ros, int T_, int hidden, float eps, int dtype,
               void* stream) {
  if (!valid_dtype(dtype)) return fail(NB_ERR_INVALID_ARG, "invalid dtype %d", dtype);
  if (!x || !w || !out || (ADD && (!res || !ro)))
    return fail(NB_ERR_INVALID_ARG, "null pointer argument");
  if (hidden <= 0 || T_ < 0) return fail(NB_ERR_INVALID_ARG, "bad sizes");
  if (xs < hidden || os < hidden || (ADD && (rs < hidden || ros < hidden)))
    return fail(NB_ERR_INVALID_ARG, "row stride smaller than hidden");
  if (T_ == 0) return NB_OK;
  if (T_ > 0x7fffffff / 2) return fail(NB_ERR_INVALID_ARG, "too many rows");
  cudaStream_t st = (cudaStream_t)stream;
  switch (dtype) {
    case NB_DTYPE_F32: return launch_norm<float, ADD>(x, xs, res, rs, w, out, os, ro, ros, T_, hidden, eps, st);
    case NB_DTYPE_F16: return launch_norm<__half, ADD>(x, xs, res, rs, w, out, os, ro, ros, T_, hidden, eps, st);
    default: return launch_norm<__nv_bfloat16, ADD>(x, xs, res, rs, w, out, os, ro, ros, T_, hidden, eps, st);
  }
}

}  // namespace nbh

extern "C" {

int nb_rmsnorm(const void* x, int64_t x_stride, const void* weight, void* out,
               int64_t out_stride, int num_tokens, int hidden, float eps, int dtype,
               void* stream) {
  return nbh::norm_entry<false>(x, x_stride, nullptr, 0, weight, out, out_stride, nullptr, 0,
                                num_tokens, hidden, eps, dtype, stream);
}

int nb_fused_add_rmsnorm(const void* x, int64_t x_stride, const void* residual,
                         int64_t residual_stride, const void* weight, void* out,
                         int64_t out_stride, void* residual_out, int64_t residual_out_stride,
                         int num_tokens, int hidden, float eps, int dtype, void* stream) {
  return nbh::norm_entry<true>(x, x_stride, residual, residual_stride, weight, out, out_stride,
                               residual_out, residual_out_stride, num_tokens, hidden, eps, dtype,
                               stream);
}

}  // extern "C"
