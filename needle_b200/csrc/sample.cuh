// Batched sampler: greedy argmax and temperature / top-k / top-p draws for a
// whole decode step in one launch.
//
// needle's Sampler.sample (needle/model/sampler.py:24-46) walks the batch row
// by row with one host read per row: int(argmax) for temperature 0, otherwise
// logit / temperature, top-k masking (logit < k-th largest -> -inf), top-p
// masking on the descending sort (a token is removed when the probability
// mass before it exceeds top_p), softmax and torch.multinomial.  Here one CTA
// takes one row:
//   * greedy rows: the first index of the maximum (NaN counts as maximal, as
//     in torch.argmax);
//   * sampled rows: x = round(logit / t) in the logits' dtype; the k-th
//     largest x by an exact radix select over order-preserving integer keys
//     (8-bit digits, most significant first); the top-p boundary by the same
//     radix select weighted by probability mass (fp32 sums), tokens of equal
//     value ordered by index (the order a stable descending sort gives);
//     then one draw by inverse CDF in vocabulary order with the caller's
//     uniform number u in [0, 1).
// Every pass re-reads the row (256 KB at a 128k vocabulary, L2-resident after
// the first).  Probabilities follow needle's rounding: each is rounded to the
// logits' dtype before it enters the mass sums.
#pragma once
#include "nb_common.cuh"

namespace nb {

constexpr int kSampleThreads = 1024;
constexpr int kBandCap = 2048;  // top-p boundary candidates sorted in shared memory

template <typename T> struct SKey;
template <> struct SKey<__nv_bfloat16> {
  using U = uint16_t;
  static constexpr int kBits = 16;
  static __device__ __forceinline__ uint32_t key(__nv_bfloat16 x) {
    const uint32_t b = __bfloat16_as_ushort(x);
    return (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
  }
};
template <> struct SKey<__half> {
  using U = uint16_t;
  static constexpr int kBits = 16;
  static __device__ __forceinline__ uint32_t key(__half x) {
    const uint32_t b = __half_as_ushort(x);
    return (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
  }
};
template <> struct SKey<float> {
  using U = uint32_t;
  static constexpr int kBits = 32;
  static __device__ __forceinline__ uint32_t key(float x) {
    const uint32_t b = __float_as_uint(x);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  }
};

// x / t rounded to the logits' dtype (torch divides a bf16/fp16 tensor by a
// Python float in fp32 and rounds once).
template <typename T>
__device__ __forceinline__ T scaled(T x, float t) {
  return Dt<T>::from_f(__fdiv_rn(Dt<T>::to_f(x), t));
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = l < (int)(blockDim.x >> 5) ? red[l] : 0.f;
  return warp_sum(s);
}

template <typename T>
__global__ void __launch_bounds__(kSampleThreads)
    sample_kernel(const T* __restrict__ logits, int64_t stride, int V,
                  const float* __restrict__ temperature, const int32_t* __restrict__ top_k,
                  const float* __restrict__ top_p, const float* __restrict__ uniforms,
                  T* __restrict__ filtered, int64_t fstride, int64_t* __restrict__ token_ids) {
  using K = SKey<T>;
  __shared__ float s_mass[256];
  __shared__ unsigned s_cnt[256];
  __shared__ float s_red[32];
  __shared__ unsigned long long s_best;
  __shared__ uint32_t s_key;
  __shared__ float s_massf;
  __shared__ unsigned s_cntf;
  __shared__ int s_tok;
  const int r = blockIdx.x, tid = threadIdx.x;
  const T* row = logits + (int64_t)r * stride;
  const float t = temperature[r];

  if (t == 0.f) {
    // greedy: the largest ordered key, then the smallest index; NaN maps
    // above every number.  A thread visits its indices in increasing order,
    // so a strictly larger key is the only update it needs.
    uint32_t bk = 0;
    int bi = 0x7FFFFFFF;
    constexpr int VEC = 16 / sizeof(T);
    auto visit = [&](T x, int i) {
      const float f = Dt<T>::to_f(x);
      const uint32_t k = f != f ? 0xFFFFFFFFu : K::key(x);
      if (k > bk || bi == 0x7FFFFFFF) {
        bk = k;
        bi = i;
      }
    };
    if (((uintptr_t)row & 15) == 0) {
      // 16-byte vectors, four in flight per thread
      const int nv = V / VEC;
      const uint4* rv = reinterpret_cast<const uint4*>(row);
      for (int v0 = tid; v0 < nv; v0 += 4 * blockDim.x) {
        uint4 buf[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int v = v0 + u * blockDim.x;
          if (v < nv) buf[u] = __ldg(rv + v);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int v = v0 + u * blockDim.x;
          if (v < nv) {
            const T* xs = reinterpret_cast<const T*>(&buf[u]);
#pragma unroll
            for (int e = 0; e < VEC; ++e) visit(xs[e], v * VEC + e);
          }
        }
      }
      for (int i = nv * VEC + tid; i < V; i += blockDim.x) visit(row[i], i);
    } else {
      for (int i = tid; i < V; i += blockDim.x) visit(row[i], i);
    }
    // (key, ~index): the block maximum is the largest key at the smallest index
    unsigned long long best =
        bi == 0x7FFFFFFF ? 0ull
                         : ((unsigned long long)bk << 32) | (uint32_t)(~(uint32_t)bi);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long b = __shfl_xor_sync(0xffffffffu, best, o);
      best = b > best ? b : best;
    }
    if (tid == 0) s_best = 0;
    __syncthreads();
    if ((tid & 31) == 0) atomicMax(&s_best, best);
    __syncthreads();
    if (tid == 0) token_ids[r] = (int64_t)(~(uint32_t)(s_best & 0xFFFFFFFFu));
    return;
  }

  // ---- top-k: key of the k-th largest scaled logit -------------------------
  uint32_t kth = 0;  // keep every key >= kth
  const int kk = top_k[r];
  if (kk > 0 && kk < V) {
    uint32_t prefix = 0;
    unsigned need = (unsigned)kk;  // rank still to find inside the current prefix
    for (int shift = K::kBits - 8; shift >= 0; shift -= 8) {
      for (int b = tid; b < 256; b += blockDim.x) s_cnt[b] = 0;
      __syncthreads();
      const uint32_t hi_mask = shift + 8 >= 32 ? 0u : (0xFFFFFFFFu << (shift + 8));
      for (int i = tid; i < V; i += blockDim.x) {
        const uint32_t k = K::key(scaled(row[i], t));
        if ((k & hi_mask) == (prefix & hi_mask)) atomicAdd(&s_cnt[(k >> shift) & 0xFF], 1u);
      }
      __syncthreads();
      if (tid == 0) {
        unsigned acc = 0;
        int b = 255;
        for (; b > 0; --b) {
          if (acc + s_cnt[b] >= need) break;
          acc += s_cnt[b];
        }
        s_key = prefix | ((uint32_t)b << shift);
        s_cntf = need - acc;
      }
      __syncthreads();
      prefix = s_key;
      need = s_cntf;
      __syncthreads();
    }
    kth = prefix;
  }

  // ---- softmax over the kept tokens (fp32; each probability rounded to T) --
  float mx = -INFINITY;
  for (int i = tid; i < V; i += blockDim.x) {
    const T x = scaled(row[i], t);
    if (K::key(x) >= kth) mx = fmaxf(mx, Dt<T>::to_f(x));
  }
  mx = warp_max(mx);
  if ((tid & 31) == 0) s_red[tid >> 5] = mx;
  __syncthreads();
  if (tid < 32) {
    float v = tid < (int)(blockDim.x >> 5) ? s_red[tid] : -INFINITY;
    v = warp_max(v);
    if (tid == 0) s_massf = v;
  }
  __syncthreads();
  mx = s_massf;
  float z = 0.f;
  for (int i = tid; i < V; i += blockDim.x) {
    const T x = scaled(row[i], t);
    if (K::key(x) >= kth) z += __expf(Dt<T>::to_f(x) - mx);
  }
  z = block_sum(z, s_red);
  const float inv_z = 1.f / z;
  auto prob = [&](T x) { return Dt<T>::round(__expf(Dt<T>::to_f(x) - mx) * inv_z); };

  // ---- top-p -----------------------------------------------------------------
  // needle removes a token when round(round(S) - p) > round(top_p) in the
  // logits' dtype, S the running fp32 sum of the rounded probabilities in
  // descending order (torch's cumsum), p the token's own probability.  The
  // rounding only matters within a couple of units in the last place of
  // top_p: tokens whose mass before them lies below that band are kept, those
  // above it removed, and the tokens in the band are sorted (value
  // descending, index ascending: a stable sort's tie order) and scanned
  // sequentially with those rounding points.  The result is a boundary value
  // pkey and a tie count: keep keys > pkey and the first n_tie tokens of
  // value pkey in index order.
  uint32_t pkey = 0;
  unsigned n_tie = 0xFFFFFFFFu;
  const float pp = top_p[r];
  const float pth = Dt<T>::round(pp);  // the comparison runs in the logits' dtype
  // the value block where the inclusive mass (from the top) first exceeds th;
  // `above` = mass of all larger values; false if the whole mass stays <= th
  auto select_mass = [&](float th, uint32_t& key, float& above) -> bool {
    uint32_t prefix = 0;
    above = 0.f;
    for (int shift = K::kBits - 8; shift >= 0; shift -= 8) {
      for (int b = tid; b < 256; b += blockDim.x) {
        s_mass[b] = 0.f;
        s_cnt[b] = 0;
      }
      __syncthreads();
      const uint32_t hi_mask = shift + 8 >= 32 ? 0u : (0xFFFFFFFFu << (shift + 8));
      for (int i = tid; i < V; i += blockDim.x) {
        const T x = scaled(row[i], t);
        const uint32_t k = K::key(x);
        if (k >= kth && (k & hi_mask) == (prefix & hi_mask)) {
          atomicAdd(&s_mass[(k >> shift) & 0xFF], prob(x));
          atomicAdd(&s_cnt[(k >> shift) & 0xFF], 1u);
        }
      }
      __syncthreads();
      if (tid == 0) {
        float acc = above;
        int b = 255;
        bool found = false;
        for (; b >= 0; --b) {
          if (!s_cnt[b]) continue;
          if (acc + s_mass[b] > th) {
            found = true;
            break;
          }
          acc += s_mass[b];
        }
        s_cntf = found ? 1u : 0u;
        s_key = found ? (prefix | ((uint32_t)b << shift)) : 0u;
        s_massf = acc;
      }
      __syncthreads();
      const bool found = s_cntf != 0;
      prefix = s_key;
      above = s_massf;
      __syncthreads();
      if (!found) return false;
    }
    key = prefix;
    return true;
  };
  __shared__ unsigned long long s_band[kBandCap];
  __shared__ unsigned s_nband;
  if (pp < 1.f) {
    // a couple of units in the last place of top_p in the logits' dtype
    const float ulp = fabsf(pth) * (K::kBits == 16 ? (__is_same(T, __half) ? 0x1p-10f : 0x1p-7f)
                                                   : 0x1p-23f);
    uint32_t kL = 0, kU = kth;
    float aL = 0.f, aU = 0.f;
    if (select_mass(pth - 2.f * ulp, kL, aL)) {
      if (!select_mass(pth + 2.f * ulp, kU, aU)) kU = kth;
      // gather the band: keys in [kU, kL]
      if (tid == 0) s_nband = 0;
      __syncthreads();
      for (int i = tid; i < V; i += blockDim.x) {
        const uint32_t k = K::key(scaled(row[i], t));
        if (k >= kth && k >= kU && k <= kL) {
          const unsigned slot = atomicAdd(&s_nband, 1u);
          if (slot < (unsigned)kBandCap)
            s_band[slot] = ((unsigned long long)k << 32) | (uint32_t)(~(uint32_t)i);
        }
      }
      __syncthreads();
      const unsigned nb = s_nband;
      if (nb <= (unsigned)kBandCap) {
        // bitonic sort, descending, over the next power of two (pads sort last)
        unsigned n2 = 1;
        while (n2 < nb) n2 <<= 1;
        for (unsigned i = nb + tid; i < n2; i += blockDim.x) s_band[i] = 0ull;
        __syncthreads();
        for (unsigned size = 2; size <= n2; size <<= 1)
          for (unsigned stride = size >> 1; stride > 0; stride >>= 1) {
            for (unsigned i = tid; i < n2; i += blockDim.x) {
              const unsigned j = i ^ stride;
              if (j > i) {
                const unsigned long long a = s_band[i], b = s_band[j];
                const bool desc = (i & size) == 0;
                if (desc ? a < b : a > b) {
                  s_band[i] = b;
                  s_band[j] = a;
                }
              }
            }
            __syncthreads();
          }
        if (tid == 0) {
          // sequential scan with needle's rounding points
          float S = aL;
          uint32_t cur = 0xFFFFFFFFu;
          unsigned rank = 0;
          uint32_t bkey = 0;
          unsigned btie = 0xFFFFFFFFu;
          bool cut = false;
          for (unsigned c = 0; c < nb; ++c) {
            const uint32_t k = (uint32_t)(s_band[c] >> 32);
            if (k != cur) {
              cur = k;
              rank = 0;
            }
            T xv;
            if constexpr (K::kBits == 16) {
              const uint16_t bits =
                  (k & 0x8000u) ? (uint16_t)(k & 0x7FFFu) : (uint16_t)(~k & 0xFFFFu);
              memcpy(&xv, &bits, 2);
            } else {
              const uint32_t bits = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
              memcpy(&xv, &bits, 4);
            }
            const float pv = prob(xv);
            S = __fadd_rn(S, pv);
            const float d = Dt<T>::round(__fsub_rn(Dt<T>::round(S), pv));
            if (d > pth) {
              bkey = k;
              btie = rank;
              cut = true;
              break;
            }
            ++rank;
          }
          if (!cut) {  // every band token kept: the cut is right below the band
            bkey = kU;
            btie = 0xFFFFFFFFu;
          }
          s_key = bkey;
          s_cntf = btie;
        }
        __syncthreads();
        pkey = s_key;
        n_tie = s_cntf;
        __syncthreads();
      } else {
        // band too wide to sort here: the fp32 criterion (mass before <= top_p)
        uint32_t kb;
        float ab;
        if (select_mass(pth, kb, ab)) {
          pkey = kb;
          T xv;
          if constexpr (K::kBits == 16) {
            const uint16_t bits =
                (kb & 0x8000u) ? (uint16_t)(kb & 0x7FFFu) : (uint16_t)(~kb & 0xFFFFu);
            memcpy(&xv, &bits, 2);
          } else {
            const uint32_t bits = (kb & 0x80000000u) ? (kb & 0x7FFFFFFFu) : ~kb;
            memcpy(&xv, &bits, 4);
          }
          const float pv = prob(xv);
          n_tie = pv > 0.f ? (unsigned)floorf((pth - ab) / pv) + 1u : 0xFFFFFFFFu;
        }
      }
    }
  }
  // kept(i): key >= kth and (key > pkey, or key == pkey and rank-in-ties < n_tie)
  // Tie ranks need an ordered count only when the tie block is cut.
  const bool cut = pp < 1.f && n_tie != 0xFFFFFFFFu;

  // ---- draw: inverse CDF in vocabulary order over contiguous chunks ---------
  const int chunk = (V + blockDim.x - 1) / blockDim.x;
  const int i0 = min(V, tid * chunk), i1 = min(V, i0 + chunk);
  // rank of this chunk's first tie token among all tie tokens (index order)
  unsigned tie_base = 0;
  if (cut) {
    unsigned c = 0;
    for (int i = i0; i < i1; ++i) c += K::key(scaled(row[i], t)) == pkey;
    // exclusive block scan of c
    unsigned inc = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned y = __shfl_up_sync(0xffffffffu, inc, o);
      if ((tid & 31) >= o) inc += y;
    }
    __syncthreads();
    if ((tid & 31) == 31) s_cnt[tid >> 5] = inc;
    __syncthreads();
    if (tid < 32) {
      unsigned w = tid < (int)(blockDim.x >> 5) ? s_cnt[tid] : 0u;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned y = __shfl_up_sync(0xffffffffu, w, o);
        if (tid >= o) w += y;
      }
      s_cnt[tid] = w;  // inclusive sums per warp
    }
    __syncthreads();
    tie_base = inc - c + ((tid >> 5) ? s_cnt[(tid >> 5) - 1] : 0u);
    __syncthreads();
  }
  auto kept = [&](uint32_t k, unsigned tie_rank) {
    if (k < kth) return false;
    if (pp < 1.f && n_tie != 0xFFFFFFFFu) {
      if (k < pkey) return false;
      if (k == pkey) return tie_rank < n_tie;
    } else if (pp < 1.f && k < pkey) {
      return false;
    }
    return true;
  };
  // kept mass of this chunk (unrounded exponentials of the filtered logits)
  float csum = 0.f;
  {
    unsigned tr = tie_base;
    for (int i = i0; i < i1; ++i) {
      const T x = scaled(row[i], t);
      const uint32_t k = K::key(x);
      const bool kp = kept(k, tr);
      tr += k == pkey;
      const float e = kp ? __expf(Dt<T>::to_f(x) - mx) : 0.f;
      csum += e;
      if (filtered) filtered[(int64_t)r * fstride + i] = kp ? x : Dt<T>::from_f(-INFINITY);
    }
  }
  // exclusive scan of the chunk sums (fp32), then the chunk holding u * total
  float inc = csum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, inc, o);
    if ((tid & 31) >= o) inc += y;
  }
  __syncthreads();
  if ((tid & 31) == 31) s_mass[tid >> 5] = inc;
  __syncthreads();
  if (tid < 32) {
    float w = tid < (int)(blockDim.x >> 5) ? s_mass[tid] : 0.f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, w, o);
      if (tid >= o) w += y;
    }
    s_mass[tid] = w;
  }
  if (tid == 0) s_tok = -1;
  __syncthreads();
  const float total = s_mass[(blockDim.x >> 5) - 1];
  const float excl = inc - csum + ((tid >> 5) ? s_mass[(tid >> 5) - 1] : 0.f);
  const float target = fminf(uniforms[r], 0.99999994f) * total;
  if (csum > 0.f && excl <= target && target < excl + csum) {
    float acc = excl;
    unsigned tr = tie_base;
    int pick = -1, last = -1;
    for (int i = i0; i < i1; ++i) {
      const T x = scaled(row[i], t);
      const uint32_t k = K::key(x);
      const bool kp = kept(k, tr);
      tr += k == pkey;
      if (!kp) continue;
      last = i;
      acc += __expf(Dt<T>::to_f(x) - mx);
      if (acc > target) {
        pick = i;
        break;
      }
    }
    atomicMax(&s_tok, pick >= 0 ? pick : last);
  }
  __syncthreads();
  if (tid == 0) {
    int tok = s_tok;
    if (tok < 0) {  // rounding at the very end of the distribution: the last kept token
      for (int i = V - 1; i >= 0; --i)
        if (K::key(scaled(row[i], t)) >= kth) { tok = i; break; }
    }
    token_ids[r] = tok;
  }
}

}  // namespace nb

extern "C" {

int nb_sample(const void* logits, int64_t row_stride, int num_rows, int vocab,
              const float* temperature, const int32_t* top_k, const float* top_p,
              const float* uniforms, void* filtered, int64_t filtered_stride,
              int64_t* token_ids, int dtype, void* stream) {
  using namespace nbh;
  if (!valid_dtype(dtype)) return fail(NB_ERR_INVALID_ARG, "invalid dtype %d", dtype);
  if (!logits || !temperature || !top_k || !top_p || !uniforms || !token_ids)
    return fail(NB_ERR_INVALID_ARG, "null pointer argument");
  if (num_rows < 0 || vocab <= 0) return fail(NB_ERR_INVALID_ARG, "bad sizes");
  if (row_stride < vocab || (filtered && filtered_stride < vocab))
    return fail(NB_ERR_INVALID_ARG, "row stride smaller than the vocabulary");
  if (num_rows == 0) return NB_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const int threads = nb::kSampleThreads;
  switch (dtype) {
    case NB_DTYPE_F32:
      nb::sample_kernel<float><<<num_rows, threads, 0, st>>>(
          (const float*)logits, row_stride, vocab, temperature, top_k, top_p, uniforms,
          (float*)filtered, filtered_stride, token_ids);
      break;
    case NB_DTYPE_F16:
      nb::sample_kernel<__half><<<num_rows, threads, 0, st>>>(
          (const __half*)logits, row_stride, vocab, temperature, top_k, top_p, uniforms,
          (__half*)filtered, filtered_stride, token_ids);
      break;
    default:
      nb::sample_kernel<__nv_bfloat16><<<num_rows, threads, 0, st>>>(
          (const __nv_bfloat16*)logits, row_stride, vocab, temperature, top_k, top_p, uniforms,
          (__nv_bfloat16*)filtered, filtered_stride, token_ids);
  }
  return check_launch("sample");
}

}  // extern "C"
