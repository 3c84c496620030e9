// store_kvcache, RoPE, and RoPE fused with the KV store.
//
// All three are HBM-bound elementwise/scatter kernels on 16-byte vectors,
// consecutive threads on consecutive vectors of one head row so that both the
// token-major reads and the cache-row writes are coalesced.  The cache writers
// give each CTA a few tokens and resolve each token's slot once, in shared
// memory, before the copy.
#pragma once
#include <algorithm>

#include "nb_common.cuh"

namespace nb {

// Slot of token i (of len new tokens) of a sequence whose context (tokens
// already cached) is c.  Restates the index math of
// needle/layers/attention.py:214-240: position = c + i, column = position /
// block_size clamped to the last table column.  Returns false (and records
// why) when the token must not be written.
__device__ __forceinline__ bool slot_of(int s, int i, int len, int c,
                                        const int32_t* __restrict__ bt, int64_t bt_stride,
                                        int maxb, int num_blocks, int block_size, int& phys,
                                        int& off) {
  const int pos = c + i;
  if (c < 0) {
    set_error(kErrPosition);
    return false;
  }
  const int col_u = pos / block_size;
  const int col = col_u < maxb - 1 ? col_u : maxb - 1;
  // Clamped tail: a later token of the same sequence lands on the same slot;
  // only the last one writes (the reference applies them in order).
  if (col_u >= maxb - 1 && pos + block_size < c + len) return false;
  phys = __ldg(bt + (int64_t)s * bt_stride + col);
  if (phys < 0 || phys >= num_blocks) {
    set_error(kErrBlockId);
    return false;
  }
  off = pos - col_u * block_size;
  return true;
}

// Slot of new token `t` (global token index): its sequence from cu_seqlens
// (prefill) or t itself (decode, cu == nullptr), then slot_of.
__device__ __forceinline__ bool token_slot(int t, const int32_t* __restrict__ cu,
                                           const int32_t* __restrict__ ctx, int num_seqs,
                                           const int32_t* __restrict__ bt, int64_t bt_stride,
                                           int maxb, int num_blocks, int block_size, int& phys,
                                           int& off) {
  int s, i, len;
  if (cu) {
    s = seq_of_token(cu, num_seqs, t);
    const int c0 = __ldg(cu + s);
    i = t - c0;
    len = __ldg(cu + s + 1) - c0;
  } else {
    s = t;
    i = 0;
    len = 1;
  }
  return slot_of(s, i, len, __ldg(ctx + s), bt, bt_stride, maxb, num_blocks, block_size, phys,
                 off);
}

constexpr int kMaxTokPerCta = 64;

constexpr int kSmemSeqs = 1024;  // cu_seqlens / context_lens staged in shared memory up to this

// Slots of this CTA's tokens [t0, t0 + nt) into shared memory (phys = -1:
// the token is not written), computed once per token instead of once per
// 16-byte vector.  For prefill batches of up to kSmemSeqs sequences the CTA
// first stages cu_seqlens and context_lens in shared memory (one cooperative
// round trip) and searches there, so a token's slot costs two dependent
// global loads (that stage, then its block-table entry) instead of a binary
// search through global memory.  kStage = false skips the staging (CTAs of a
// single token, where the stage costs more than the search).
template <bool kStage>
__device__ __forceinline__ void cta_token_slots(int t0, int nt, const int32_t* __restrict__ cu,
                                                const int32_t* __restrict__ ctx, int num_seqs,
                                                const int32_t* __restrict__ bt,
                                                int64_t bt_stride, int maxb, int num_blocks,
                                                int block_size, int* s_phys, int* s_off) {
  __shared__ int s_cu[kSmemSeqs + 1];
  __shared__ int s_ctx[kSmemSeqs];
  if (kStage && cu != nullptr && num_seqs <= kSmemSeqs) {  // uniform over the CTA
    for (int i = threadIdx.x; i <= num_seqs; i += blockDim.x) {
      s_cu[i] = __ldg(cu + i);
      if (i < num_seqs) s_ctx[i] = __ldg(ctx + i);
    }
    __syncthreads();
    if (threadIdx.x < nt) {
      const int t = t0 + threadIdx.x;
      int lo = 0, hi = num_seqs - 1;  // last sequence whose start is <= t
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (s_cu[mid] <= t) lo = mid; else hi = mid - 1;
      }
      int phys = -1, off = 0;
      if (!slot_of(lo, t - s_cu[lo], s_cu[lo + 1] - s_cu[lo], s_ctx[lo], bt, bt_stride, maxb,
                   num_blocks, block_size, phys, off))
        phys = -1;
      s_phys[threadIdx.x] = phys;
      s_off[threadIdx.x] = off;
    }
  } else if (threadIdx.x < nt) {
    int phys = -1, off = 0;
    if (!token_slot(t0 + threadIdx.x, cu, ctx, num_seqs, bt, bt_stride, maxb, num_blocks,
                    block_size, phys, off))
      phys = -1;
    s_phys[threadIdx.x] = phys;
    s_off[threadIdx.x] = off;
  }
  __syncthreads();
}

// K/V rows of tok_per_cta tokens per CTA.  Items are 16-byte vectors ordered
// (token, head, K/V, vector) so consecutive threads read consecutive vectors
// of a token row and write consecutive vectors of a cache row.  The sources
// do not depend on the slots: every thread issues its first U loads, then the
// CTA resolves its tokens' slots while those loads are in flight, then stores.
template <typename T>
__global__ void __launch_bounds__(256)
    store_kvcache_kernel(const T* __restrict__ k, int64_t k_stride, const T* __restrict__ v,
                         int64_t v_stride, T* __restrict__ cache, int num_blocks, int kvh,
                         int block_size, int D, const int32_t* __restrict__ bt, int64_t bt_stride,
                         int maxb, const int32_t* __restrict__ cu, const int32_t* __restrict__ ctx,
                         int num_seqs, int num_tokens, int tok_per_cta) {
  griddep_launch_dependents();  // the paged decode that follows may start its launch
  __shared__ int s_phys[kMaxTokPerCta], s_off[kMaxTokPerCta];
  constexpr int VEC = 16 / sizeof(T);
  constexpr int U = 4;
  const int vpr = D / VEC;  // vectors per head row
  const int t0 = blockIdx.x * tok_per_cta;
  const int nt = min(tok_per_cta, num_tokens - t0);
  const int items = nt * kvh * 2 * vpr;
  uint4 val[U];
  auto load = [&](int base) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int idx = base + u * blockDim.x;
      if (idx < items) {
        const int vec = idx % vpr;
        int r = idx / vpr;
        const int which = r & 1;  // 0 = K, 1 = V
        r >>= 1;
        const int64_t t = t0 + r / kvh;
        const T* src = (which ? v + t * v_stride : k + t * k_stride) + (int64_t)(r % kvh) * D +
                       vec * VEC;
        val[u] = __ldg(reinterpret_cast<const uint4*>(src));
      }
    }
  };
  auto store = [&](int base) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int idx = base + u * blockDim.x;
      if (idx < items) {
        const int vec = idx % vpr;
        int r = idx / vpr;
        const int which = r & 1;
        r >>= 1;
        const int h = r % kvh, lt = r / kvh;
        const int phys = s_phys[lt];
        if (phys >= 0)
          *reinterpret_cast<uint4*>(
              cache + ((((int64_t)which * num_blocks + phys) * kvh + h) * block_size + s_off[lt]) * D +
              vec * VEC) = val[u];
      }
    }
  };
  load(threadIdx.x);
  cta_token_slots<true>(t0, nt, cu, ctx, num_seqs, bt, bt_stride, maxb, num_blocks, block_size, s_phys,
                  s_off);
  store(threadIdx.x);
  for (int base = threadIdx.x + U * blockDim.x; base < items; base += U * blockDim.x) {
    load(base);
    store(base);
  }
}

// Scalar fallback for shapes whose rows are not 16-byte vectorisable.
template <typename T>
__global__ void __launch_bounds__(256)
    store_kvcache_scalar_kernel(const T* __restrict__ k, int64_t k_stride,
                                const T* __restrict__ v, int64_t v_stride, T* __restrict__ cache,
                                int num_blocks, int kvh, int block_size, int D,
                                const int32_t* __restrict__ bt, int64_t bt_stride, int maxb,
                                const int32_t* __restrict__ cu, const int32_t* __restrict__ ctx,
                                int num_seqs, int num_tokens) {
  const int64_t total = (int64_t)num_tokens * kvh * 2 * D;
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= total) return;
  const int e = (int)(gid % D);
  int64_t r = gid / D;
  const int which = (int)(r & 1);
  r >>= 1;
  const int h = (int)(r % kvh);
  const int t = (int)(r / kvh);
  int phys, off;
  if (!token_slot(t, cu, ctx, num_seqs, bt, bt_stride, maxb, num_blocks, block_size, phys, off))
    return;
  const T* src = (which ? v + (int64_t)t * v_stride : k + (int64_t)t * k_stride) + (int64_t)h * D;
  cache[((((int64_t)which * num_blocks + phys) * kvh + h) * block_size + off) * D + e] = src[e];
}

// One rotation step of needle/layers/attention.py:277-288 for the element
// pair (x_lo = x[i], x_hi = x[i + D/2]):
//   out[i]       = rnd(rnd(x_lo * cos[i])       + rnd(-x_hi * sin[i]))
//   out[i + D/2] = rnd(rnd(x_hi * cos[i + D/2]) + rnd( x_lo * sin[i + D/2]))
// rnd rounds to the storage type after every op, like torch's elementwise
// kernels; __fmul_rn/__fadd_rn keep the fp32 case free of FMA contraction.
template <typename T>
__device__ __forceinline__ void rope_pair(float xl, float xh, float cl, float ch, float sl,
                                          float sh, float& ol, float& oh) {
  const float a = Dt<T>::round(__fmul_rn(xl, cl));
  const float b = Dt<T>::round(__fmul_rn(-xh, sl));
  ol = Dt<T>::round(__fadd_rn(a, b));
  const float c = Dt<T>::round(__fmul_rn(xh, ch));
  const float d = Dt<T>::round(__fmul_rn(xl, sh));
  oh = Dt<T>::round(__fadd_rn(c, d));
}

// Rotate VEC element pairs of one head row in place.
template <typename T, int VEC>
__device__ __forceinline__ void rope_row_vec(T* row, const T* __restrict__ cs,
                                             const T* __restrict__ sn, int half, int j) {
  // j: first element of this thread's chunk in [0, half)
  T lo[VEC], hi[VEC], cl[VEC], ch[VEC], sl[VEC], sh[VEC];
  if constexpr (VEC * sizeof(T) == 16) {
    *reinterpret_cast<uint4*>(lo) = *reinterpret_cast<const uint4*>(row + j);
    *reinterpret_cast<uint4*>(hi) = *reinterpret_cast<const uint4*>(row + j + half);
    *reinterpret_cast<uint4*>(cl) = __ldg(reinterpret_cast<const uint4*>(cs + j));
    *reinterpret_cast<uint4*>(ch) = __ldg(reinterpret_cast<const uint4*>(cs + j + half));
    *reinterpret_cast<uint4*>(sl) = __ldg(reinterpret_cast<const uint4*>(sn + j));
    *reinterpret_cast<uint4*>(sh) = __ldg(reinterpret_cast<const uint4*>(sn + j + half));
  } else {
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      lo[e] = row[j + e]; hi[e] = row[j + half + e];
      cl[e] = cs[j + e]; ch[e] = cs[j + half + e];
      sl[e] = sn[j + e]; sh[e] = sn[j + half + e];
    }
  }
#pragma unroll
  for (int e = 0; e < VEC; ++e) {
    float ol, oh;
    rope_pair<T>(Dt<T>::to_f(lo[e]), Dt<T>::to_f(hi[e]), Dt<T>::to_f(cl[e]), Dt<T>::to_f(ch[e]),
                 Dt<T>::to_f(sl[e]), Dt<T>::to_f(sh[e]), ol, oh);
    lo[e] = Dt<T>::from_f(ol);
    hi[e] = Dt<T>::from_f(oh);
  }
  if constexpr (VEC * sizeof(T) == 16) {
    *reinterpret_cast<uint4*>(row + j) = *reinterpret_cast<uint4*>(lo);
    *reinterpret_cast<uint4*>(row + j + half) = *reinterpret_cast<uint4*>(hi);
  } else {
#pragma unroll
    for (int e = 0; e < VEC; ++e) { row[j + e] = lo[e]; row[j + half + e] = hi[e]; }
  }
}

// In-place RoPE of q [T, Hq, D] and k [T, Hkv, D].  One thread per VEC pairs.
template <typename T, int VEC>
__global__ void __launch_bounds__(256)
    rope_kernel(T* q, int64_t q_stride, int hq, T* k, int64_t k_stride, int hk,
                const T* __restrict__ cos, const T* __restrict__ sin, int64_t cs_stride,
                int num_tokens, int D) {
  const int half = D / 2;
  const int cpr = half / VEC;                    // chunks per head row
  const int heads = hq + hk;
  const int64_t total = (int64_t)num_tokens * heads * cpr;
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= total) return;
  const int c = (int)(gid % cpr);
  const int64_t r = gid / cpr;
  const int hh = (int)(r % heads);
  const int t = (int)(r / heads);
  T* row = hh < hq ? q + (int64_t)t * q_stride + (int64_t)hh * D
                   : k + (int64_t)t * k_stride + (int64_t)(hh - hq) * D;
  rope_row_vec<T, VEC>(row, cos + (int64_t)t * cs_stride, sin + (int64_t)t * cs_stride, half,
                       c * VEC);
}

// Load / store VEC consecutive elements (one 16-byte vector when VEC fills one).
template <typename T, int VEC>
__device__ __forceinline__ void ld_chunk(T (&x)[VEC], const T* p) {
  if constexpr (VEC * sizeof(T) == 16) {
    *reinterpret_cast<uint4*>(x) = *reinterpret_cast<const uint4*>(p);
  } else {
#pragma unroll
    for (int e = 0; e < VEC; ++e) x[e] = p[e];
  }
}
template <typename T, int VEC>
__device__ __forceinline__ void st_chunk(T* p, const T (&x)[VEC]) {
  if constexpr (VEC * sizeof(T) == 16) {
    *reinterpret_cast<uint4*>(p) = *reinterpret_cast<const uint4*>(x);
  } else {
#pragma unroll
    for (int e = 0; e < VEC; ++e) p[e] = x[e];
  }
}

// RoPE of q (in place) and k, then K/V into the cache, tok_per_cta tokens per
// CTA.  Items are (token, head slot, chunk) with head slots [0, Hq) = q,
// [Hq, Hq+Hkv) = k and [Hq+Hkv, Hq+2Hkv) = v; a chunk is VEC element pairs
// (x[j..j+VEC), x[j+D/2..j+D/2+VEC)).  q chunks are rotated and written back
// at once; k/v chunks are loaded (k rotated) before the CTA resolves its
// tokens' slots, and stored to the cache after.
template <typename T, int VEC>
__global__ void __launch_bounds__(256)
    rope_store_kernel(T* q, int64_t q_stride, int hq, T* k, int64_t k_stride,
                      const T* __restrict__ v, int64_t v_stride, const T* __restrict__ cos,
                      const T* __restrict__ sin, int64_t cs_stride, T* __restrict__ cache,
                      int num_blocks, int hk, int block_size, int D,
                      const int32_t* __restrict__ bt, int64_t bt_stride, int maxb,
                      const int32_t* __restrict__ cu, const int32_t* __restrict__ ctx,
                      int num_seqs, int num_tokens, int write_k_back, int tok_per_cta) {
  griddep_launch_dependents();  // the paged decode that follows may start its launch
  __shared__ int s_phys[kMaxTokPerCta], s_off[kMaxTokPerCta];
  constexpr int U = 1;  // one chunk per thread: more threads in flight beat deeper ones here
  const int half = D / 2;
  const int cpr = half / VEC;
  const int heads = hq + 2 * hk;
  const int t0 = blockIdx.x * tok_per_cta;
  const int nt = min(tok_per_cta, num_tokens - t0);
  const int items = nt * heads * cpr;
  T lo[U][VEC], hi[U][VEC];
  auto load = [&](int base) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int idx = base + u * blockDim.x;
      if (idx >= items) continue;
      const int c = idx % cpr;
      const int r = idx / cpr;
      const int hh = r % heads;
      const int64_t t = t0 + r / heads;
      const int j = c * VEC;
      if (hh < hq) {
        rope_row_vec<T, VEC>(q + t * q_stride + (int64_t)hh * D, cos + t * cs_stride,
                             sin + t * cs_stride, half, j);
      } else if (hh < hq + hk) {
        T* row = k + t * k_stride + (int64_t)(hh - hq) * D;
        const T* cs = cos + t * cs_stride;
        const T* sn = sin + t * cs_stride;
        T cl[VEC], ch[VEC], sl[VEC], sh[VEC];
        ld_chunk<T, VEC>(lo[u], row + j);
        ld_chunk<T, VEC>(hi[u], row + j + half);
        ld_chunk<T, VEC>(cl, cs + j);
        ld_chunk<T, VEC>(ch, cs + j + half);
        ld_chunk<T, VEC>(sl, sn + j);
        ld_chunk<T, VEC>(sh, sn + j + half);
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          float ol, oh;
          rope_pair<T>(Dt<T>::to_f(lo[u][e]), Dt<T>::to_f(hi[u][e]), Dt<T>::to_f(cl[e]),
                       Dt<T>::to_f(ch[e]), Dt<T>::to_f(sl[e]), Dt<T>::to_f(sh[e]), ol, oh);
          lo[u][e] = Dt<T>::from_f(ol);
          hi[u][e] = Dt<T>::from_f(oh);
        }
        if (write_k_back) {
          st_chunk<T, VEC>(row + j, lo[u]);
          st_chunk<T, VEC>(row + j + half, hi[u]);
        }
      } else {
        const T* row = v + t * v_stride + (int64_t)(hh - hq - hk) * D;
        ld_chunk<T, VEC>(lo[u], row + j);
        ld_chunk<T, VEC>(hi[u], row + j + half);
      }
    }
  };
  auto store = [&](int base) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int idx = base + u * blockDim.x;
      if (idx >= items) continue;
      const int c = idx % cpr;
      const int r = idx / cpr;
      const int hh = r % heads;
      const int lt = r / heads;
      if (hh < hq) continue;
      const bool is_k = hh < hq + hk;
      const int h = is_k ? hh - hq : hh - hq - hk;
      const int phys = s_phys[lt];
      if (phys < 0) continue;
      T* dst = cache +
               ((((int64_t)(is_k ? 0 : 1) * num_blocks + phys) * hk + h) * block_size + s_off[lt]) *
                   D +
               c * VEC;
      st_chunk<T, VEC>(dst, lo[u]);
      st_chunk<T, VEC>(dst + half, hi[u]);
    }
  };
  load(threadIdx.x);
  cta_token_slots<false>(t0, nt, cu, ctx, num_seqs, bt, bt_stride, maxb, num_blocks, block_size, s_phys,
                  s_off);
  store(threadIdx.x);
  for (int base = threadIdx.x + U * blockDim.x; base < items; base += U * blockDim.x) {
    load(base);
    store(base);
  }
}

}  // namespace nb

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
namespace nbh {

inline int check_cache_args(const void* cache, int num_blocks, int kvh, int block_size, int D,
                            const int32_t* bt, int64_t bt_stride, int maxb,
                            const int32_t* ctx, int num_seqs, int num_tokens) {
  if (!cache || !bt || !ctx) return fail(NB_ERR_INVALID_ARG, "null cache/block_table/context_lens");
  if (num_blocks <= 0 || kvh <= 0 || block_size <= 0 || D <= 0 || maxb <= 0)
    return fail(NB_ERR_INVALID_ARG, "non-positive cache dimension");
  if (num_seqs < 0 || num_tokens < 0) return fail(NB_ERR_INVALID_ARG, "negative size");
  if (bt_stride < maxb) return fail(NB_ERR_INVALID_ARG, "block_table_stride < max_blocks_per_seq");
  return NB_OK;
}

template <typename T>
int launch_store(const void* k, int64_t ks, const void* v, int64_t vs, void* cache, int nblk,
                 int kvh, int bs, int D, const int32_t* bt, int64_t bts, int maxb,
                 const int32_t* cu, const int32_t* ctx, int nseq, int ntok, cudaStream_t st) {
  constexpr int VEC = 16 / sizeof(T);
  const bool vec_ok = (D % VEC == 0) && (ks % VEC == 0) && (vs % VEC == 0) &&
                      ((uintptr_t)k % 16 == 0) && ((uintptr_t)v % 16 == 0) &&
                      ((uintptr_t)cache % 16 == 0);
  const int threads = 256;
  if (vec_ok) {
    // about 1024 vectors (4 per thread) per CTA
    const int per_tok = kvh * 2 * (D / VEC);
    const int tok = std::max(1, std::min(nb::kMaxTokPerCta, 1024 / std::max(1, per_tok)));
    const int64_t blocks = ((int64_t)ntok + tok - 1) / tok;
    nb::store_kvcache_kernel<T><<<(unsigned)blocks, threads, 0, st>>>(
        (const T*)k, ks, (const T*)v, vs, (T*)cache, nblk, kvh, bs, D, bt, bts, maxb, cu, ctx,
        nseq, ntok, tok);
  } else {
    const int64_t total = (int64_t)ntok * kvh * 2 * D;
    const int64_t blocks = (total + threads - 1) / threads;
    nb::store_kvcache_scalar_kernel<T><<<(unsigned)blocks, threads, 0, st>>>(
        (const T*)k, ks, (const T*)v, vs, (T*)cache, nblk, kvh, bs, D, bt, bts, maxb, cu, ctx,
        nseq, ntok);
  }
  return check_launch("store_kvcache");
}

template <typename T, int VEC>
int launch_rope(void* q, int64_t qs, int hq, void* k, int64_t ks, int hk, const void* cos,
                const void* sin, int64_t css, int ntok, int D, cudaStream_t st) {
  const int64_t total = (int64_t)ntok * (hq + hk) * (D / 2 / VEC);
  const int threads = 256;
  nb::rope_kernel<T, VEC><<<(unsigned)((total + threads - 1) / threads), threads, 0, st>>>(
      (T*)q, qs, hq, (T*)k, ks, hk, (const T*)cos, (const T*)sin, css, ntok, D);
  return check_launch("rope");
}

template <typename T>
int dispatch_rope(void* q, int64_t qs, int hq, void* k, int64_t ks, int hk, const void* cos,
                  const void* sin, int64_t css, int ntok, int D, cudaStream_t st) {
  constexpr int V16 = 16 / sizeof(T);
  const bool vec_ok = ((D / 2) % V16 == 0) && (qs % V16 == 0) && (!k || ks % V16 == 0) &&
                      (css % V16 == 0) && ((uintptr_t)q % 16 == 0) &&
                      ((uintptr_t)k % 16 == 0) && ((uintptr_t)cos % 16 == 0) &&
                      ((uintptr_t)sin % 16 == 0);
  if (vec_ok) return launch_rope<T, V16>(q, qs, hq, k, ks, hk, cos, sin, css, ntok, D, st);
  return launch_rope<T, 1>(q, qs, hq, k, ks, hk, cos, sin, css, ntok, D, st);
}

template <typename T>
int launch_rope_store(void* q, int64_t qs, int hq, void* k, int64_t ks, const void* v, int64_t vs,
                      const void* cos, const void* sin, int64_t css, void* cache, int nblk,
                      int hk, int bs, int D, const int32_t* bt, int64_t bts, int maxb,
                      const int32_t* cu, const int32_t* ctx, int nseq, int ntok, int wkb,
                      cudaStream_t st) {
  if (D % 2) return fail(NB_ERR_UNSUPPORTED, "head_dim %d is odd", D);
  // 16-byte chunks when every row and table is 16-byte aligned, else scalar.
  constexpr int V16 = 16 / sizeof(T);
  const bool vec_ok = ((D / 2) % V16 == 0) && (qs % V16 == 0) && (ks % V16 == 0) &&
                      (vs % V16 == 0) && (css % V16 == 0) && ((uintptr_t)q % 16 == 0) &&
                      ((uintptr_t)k % 16 == 0) && ((uintptr_t)v % 16 == 0) &&
                      ((uintptr_t)cos % 16 == 0) && ((uintptr_t)sin % 16 == 0) &&
                      ((uintptr_t)cache % 16 == 0);
  const int threads = 256;
  auto launch = [&](auto kern, int vec) {
    // about 256 chunks (one per thread) per CTA
    const int per_tok = (hq + 2 * hk) * (D / 2 / vec);
    const int tok = std::max(1, std::min(nb::kMaxTokPerCta, 256 / std::max(1, per_tok)));
    const int64_t blocks = ((int64_t)ntok + tok - 1) / tok;
    kern<<<(unsigned)blocks, threads, 0, st>>>((T*)q, qs, hq, (T*)k, ks, (const T*)v, vs,
                                               (const T*)cos, (const T*)sin, css, (T*)cache, nblk,
                                               hk, bs, D, bt, bts, maxb, cu, ctx, nseq, ntok, wkb,
                                               tok);
    return check_launch("rope_store_kvcache");
  };
  if (vec_ok) return launch(nb::rope_store_kernel<T, V16>, V16);
  return launch(nb::rope_store_kernel<T, 1>, 1);
}

}  // namespace nbh

extern "C" {

int nb_store_kvcache(const void* k, int64_t k_stride, const void* v, int64_t v_stride,
                     void* kv_cache, int num_blocks, int num_kv_heads, int block_size,
                     int head_dim, const int32_t* block_table, int64_t block_table_stride,
                     int max_blocks_per_seq, const int32_t* cu_seqlens,
                     const int32_t* context_lens, int num_seqs, int num_tokens, int dtype,
                     void* stream) {
  using namespace nbh;
  if (!valid_dtype(dtype)) return fail(NB_ERR_INVALID_ARG, "invalid dtype %d", dtype);
  int rc = check_cache_args(kv_cache, num_blocks, num_kv_heads, block_size, head_dim, block_table,
                            block_table_stride, max_blocks_per_seq, context_lens, num_seqs,
                            num_tokens);
  if (rc) return rc;
  if (!k || !v) return fail(NB_ERR_INVALID_ARG, "null k/v");
  if (k_stride < (int64_t)num_kv_heads * head_dim || v_stride < (int64_t)num_kv_heads * head_dim)
    return fail(NB_ERR_INVALID_ARG, "k/v row stride smaller than num_kv_heads * head_dim");
  if (!cu_seqlens && num_tokens != num_seqs)
    return fail(NB_ERR_INVALID_ARG, "cu_seqlens NULL requires num_tokens == num_seqs");
  if (num_tokens == 0) return NB_OK;
  if (num_seqs == 0) return fail(NB_ERR_INVALID_ARG, "tokens without sequences");
  cudaStream_t st = (cudaStream_t)stream;
  switch (dtype) {
    case NB_DTYPE_F32:
      return launch_store<float>(k, k_stride, v, v_stride, kv_cache, num_blocks, num_kv_heads,
                                 block_size, head_dim, block_table, block_table_stride,
                                 max_blocks_per_seq, cu_seqlens, context_lens, num_seqs,
                                 num_tokens, st);
    case NB_DTYPE_F16:
      return launch_store<__half>(k, k_stride, v, v_stride, kv_cache, num_blocks, num_kv_heads,
                                  block_size, head_dim, block_table, block_table_stride,
                                  max_blocks_per_seq, cu_seqlens, context_lens, num_seqs,
                                  num_tokens, st);
    default:
      return launch_store<__nv_bfloat16>(k, k_stride, v, v_stride, kv_cache, num_blocks,
                                         num_kv_heads, block_size, head_dim, block_table,
                                         block_table_stride, max_blocks_per_seq, cu_seqlens,
                                         context_lens, num_seqs, num_tokens, st);
  }
}

int nb_rope(void* q, int64_t q_stride, int num_q_heads, void* k, int64_t k_stride,
            int num_kv_heads, const void* cos, const void* sin, int64_t cs_stride, int num_tokens,
            int head_dim, int dtype, void* stream) {
  using namespace nbh;
  if (!valid_dtype(dtype)) return fail(NB_ERR_INVALID_ARG, "invalid dtype %d", dtype);
  if (!q || !cos || !sin) return fail(NB_ERR_INVALID_ARG, "null q/cos/sin");
  if (head_dim <= 0 || head_dim % 2) return fail(NB_ERR_INVALID_ARG, "head_dim must be even");
  if (num_q_heads <= 0 || num_tokens < 0) return fail(NB_ERR_INVALID_ARG, "bad sizes");
  if (!k) num_kv_heads = 0;
  if (k && num_kv_heads <= 0) return fail(NB_ERR_INVALID_ARG, "num_kv_heads must be > 0");
  if (q_stride < (int64_t)num_q_heads * head_dim ||
      (k && k_stride < (int64_t)num_kv_heads * head_dim) || cs_stride < head_dim)
    return fail(NB_ERR_INVALID_ARG, "row stride too small");
  if (num_tokens == 0) return NB_OK;
  cudaStream_t st = (cudaStream_t)stream;
  switch (dtype) {
    case NB_DTYPE_F32:
      return dispatch_rope<float>(q, q_stride, num_q_heads, k, k_stride, num_kv_heads, cos, sin,
                                  cs_stride, num_tokens, head_dim, st);
    case NB_DTYPE_F16:
      return dispatch_rope<__half>(q, q_stride, num_q_heads, k, k_stride, num_kv_heads, cos, sin,
                                   cs_stride, num_tokens, head_dim, st);
    default:
      return dispatch_rope<__nv_bfloat16>(q, q_stride, num_q_heads, k, k_stride, num_kv_heads,
                                          cos, sin, cs_stride, num_tokens, head_dim, st);
  }
}

int nb_rope_store_kvcache(void* q, int64_t q_stride, int num_q_heads, void* k, int64_t k_stride,
                          const void* v, int64_t v_stride, const void* cos, const void* sin,
                          int64_t cs_stride, void* kv_cache, int num_blocks, int num_kv_heads,
                          int block_size, int head_dim, const int32_t* block_table,
                          int64_t block_table_stride, int max_blocks_per_seq,
                          const int32_t* cu_seqlens, const int32_t* context_lens, int num_seqs,
                          int num_tokens, int write_k_back, int dtype, void* stream) {
  using namespace nbh;
  if (!valid_dtype(dtype)) return fail(NB_ERR_INVALID_ARG, "invalid dtype %d", dtype);
  int rc = check_cache_args(kv_cache, num_blocks, num_kv_heads, block_size, head_dim, block_table,
                            block_table_stride, max_blocks_per_seq, context_lens, num_seqs,
                            num_tokens);
  if (rc) return rc;
  if (!q || !k || !v || !cos || !sin) return fail(NB_ERR_INVALID_ARG, "null q/k/v/cos/sin");
  if (head_dim % 2) return fail(NB_ERR_INVALID_ARG, "head_dim must be even");
  if (num_q_heads <= 0) return fail(NB_ERR_INVALID_ARG, "num_q_heads must be > 0");
  if (q_stride < (int64_t)num_q_heads * head_dim ||
      k_stride < (int64_t)num_kv_heads * head_dim ||
      v_stride < (int64_t)num_kv_heads * head_dim || cs_stride < head_dim)
    return fail(NB_ERR_INVALID_ARG, "row stride too small");
  if (!cu_seqlens && num_tokens != num_seqs)
    return fail(NB_ERR_INVALID_ARG, "cu_seqlens NULL requires num_tokens == num_seqs");
  if (num_tokens == 0) return NB_OK;
  if (num_seqs == 0) return fail(NB_ERR_INVALID_ARG, "tokens without sequences");
  cudaStream_t st = (cudaStream_t)stream;
  switch (dtype) {
    case NB_DTYPE_F32:
      return launch_rope_store<float>(q, q_stride, num_q_heads, k, k_stride, v, v_stride, cos,
                                      sin, cs_stride, kv_cache, num_blocks, num_kv_heads,
                                      block_size, head_dim, block_table, block_table_stride,
                                      max_blocks_per_seq, cu_seqlens, context_lens, num_seqs,
                                      num_tokens, write_k_back, st);
    case NB_DTYPE_F16:
      return launch_rope_store<__half>(q, q_stride, num_q_heads, k, k_stride, v, v_stride, cos,
                                       sin, cs_stride, kv_cache, num_blocks, num_kv_heads,
                                       block_size, head_dim, block_table, block_table_stride,
                                       max_blocks_per_seq, cu_seqlens, context_lens, num_seqs,
                                       num_tokens, write_k_back, st);
    default:
      return launch_rope_store<__nv_bfloat16>(
          q, q_stride, num_q_heads, k, k_stride, v, v_stride, cos, sin, cs_stride, kv_cache,
          num_blocks, num_kv_heads, block_size, head_dim, block_table, block_table_stride,
          max_blocks_per_seq, cu_seqlens, context_lens, num_seqs, num_tokens, write_k_back, st);
  }
}

}  // extern "C"
