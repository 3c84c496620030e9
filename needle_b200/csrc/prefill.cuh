// Causal prefill attention over each sequence's new tokens (SIMT path).
//
// One warp per (query token, query head); a CTA holds 4 consecutive queries
// of one head, so they stream the same keys through L1.  Online softmax in
// base 2 with shuffle-reduced dot products.  This path is exact enough for
// the fp32 configurations and is the fallback for shapes the tensor-core
// prefill does not take.
#pragma once
#include "nb_common.cuh"

namespace nb {

template <typename T, int D>
__global__ void __launch_bounds__(128)
    prefill_simt_kernel(const T* __restrict__ q, int64_t qs, const T* __restrict__ k, int64_t ks,
                        const T* __restrict__ v, int64_t vs, int hq, int group,
                        const int32_t* __restrict__ cu, float scale_log2, T* __restrict__ out,
                        int64_t os) {
  constexpr int EPL = D / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z, head = blockIdx.y;
  const int s0 = __ldg(cu + b), len = __ldg(cu + b + 1) - s0;
  const int i = blockIdx.x * 4 + warp;
  if (i >= len) return;
  const int kh = head / group;
  const int tq = s0 + i;
  float qv[EPL], acc[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    qv[e] = Dt<T>::to_f(q[(int64_t)tq * qs + (int64_t)head * D + lane * EPL + e]);
    acc[e] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  for (int j = 0; j <= i; ++j) {
    const int64_t tk = s0 + j;
    const T* kr = k + tk * ks + (int64_t)kh * D + lane * EPL;
    const T* vr = v + tk * vs + (int64_t)kh * D + lane * EPL;
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) s = fmaf(qv[e], Dt<T>::to_f(kr[e]), s);
    s = warp_sum(s) * scale_log2;
    const float mn = fmaxf(m, s);
    const float al = exp2f(m - mn);
    const float p = exp2f(s - mn);
    l = l * al + p;
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc[e] = fmaf(acc[e], al, p * Dt<T>::to_f(vr[e]));
    m = mn;
  }
  const float inv = 1.f / l;
#pragma unroll
  for (int e = 0; e < EPL; ++e)
    out[(int64_t)tq * os + (int64_t)head * D + lane * EPL + e] = Dt<T>::from_f(acc[e] * inv);
}

}  // namespace nb

namespace nbh {

template <typename T, int D>
int launch_prefill_simt(const void* q, int64_t qs, const void* k, int64_t ks, const void* v,
                        int64_t vs, int hq, int group, const int32_t* cu, int B, int max_seqlen,
                        float sl2, void* out, int64_t os, cudaStream_t st) {
  dim3 grid((max_seqlen + 3) / 4, hq, B);
  nb::prefill_simt_kernel<T, D><<<grid, 128, 0, st>>>((const T*)q, qs, (const T*)k, ks,
                                                      (const T*)v, vs, hq, group, cu, sl2,
                                                      (T*)out, os);
  return check_launch("prefill_simt");
}

template <typename T>
int launch_prefill_simt_d(int D, const void* q, int64_t qs, const void* k, int64_t ks,
                          const void* v, int64_t vs, int hq, int group, const int32_t* cu, int B,
                          int msl, float sl2, void* out, int64_t os, cudaStream_t st) {
  switch (D) {
    case 32: return launch_prefill_simt<T, 32>(q, qs, k, ks, v, vs, hq, group, cu, B, msl, sl2, out, os, st);
    case 64: return launch_prefill_simt<T, 64>(q, qs, k, ks, v, vs, hq, group, cu, B, msl, sl2, out, os, st);
    case 96: return launch_prefill_simt<T, 96>(q, qs, k, ks, v, vs, hq, group, cu, B, msl, sl2, out, os, st);
    case 128: return launch_prefill_simt<T, 128>(q, qs, k, ks, v, vs, hq, group, cu, B, msl, sl2, out, os, st);
    case 256: return launch_prefill_simt<T, 256>(q, qs, k, ks, v, vs, hq, group, cu, B, msl, sl2, out, os, st);
    default: return fail(NB_ERR_UNSUPPORTED, "head_dim %d not supported by prefill", D);
  }
}

}  // namespace nbh

extern "C" {

int nb_prefill_attention(const void* q, int64_t q_stride, const void* k, int64_t k_stride,
                         const void* v, int64_t v_stride, int num_q_heads, int num_kv_heads,
                         int head_dim, const int32_t* cu_seqlens, int num_seqs, int num_tokens,
                         int max_seqlen, float scale, void* out, int64_t out_stride, int dtype,
                         void* stream) {
  using namespace nbh;
  if (!valid_dtype(dtype)) return fail(NB_ERR_INVALID_ARG, "invalid dtype %d", dtype);
  if (!q || !k || !v || !cu_seqlens || !out) return fail(NB_ERR_INVALID_ARG, "null pointer");
  if (num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 || num_seqs < 0 || num_tokens < 0)
    return fail(NB_ERR_INVALID_ARG, "bad sizes");
  if (num_q_heads % num_kv_heads)
    return fail(NB_ERR_INVALID_ARG, "num_q_heads not a multiple of num_kv_heads");
  if (q_stride < (int64_t)num_q_heads * head_dim || k_stride < (int64_t)num_kv_heads * head_dim ||
      v_stride < (int64_t)num_kv_heads * head_dim || out_stride < (int64_t)num_q_heads * head_dim)
    return fail(NB_ERR_INVALID_ARG, "row stride too small");
  if (num_seqs == 0 || num_tokens == 0) return NB_OK;
  if (max_seqlen <= 0) return fail(NB_ERR_INVALID_ARG, "max_seqlen must be > 0");
  const int group = num_q_heads / num_kv_heads;
  const float sl2 = scale * nb::kLog2e;
  cudaStream_t st = (cudaStream_t)stream;
  switch (dtype) {
    case NB_DTYPE_F32: return launch_prefill_simt_d<float>(head_dim, q, q_stride, k, k_stride, v, v_stride, num_q_heads, group, cu_seqlens, num_seqs, max_seqlen, sl2, out, out_stride, st);
    case NB_DTYPE_F16: return launch_prefill_simt_d<__half>(head_dim, q, q_stride, k, k_stride, v, v_stride, num_q_heads, group, cu_seqlens, num_seqs, max_seqlen, sl2, out, out_stride, st);
    default: return launch_prefill_simt_d<__nv_bfloat16>(head_dim, q, q_stride, k, k_stride, v, v_stride, num_q_heads, group, cu_seqlens, num_seqs, max_seqlen, sl2, out, out_stride, st);
  }
}

}  // extern "C"
