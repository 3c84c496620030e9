// Slot table of one forward and the KV writers that read it.
//
// Every layer of a step writes its new K/V rows to the same cache positions:
// token t of sequence s goes to position context_lens[s] + i, whose block is
// block_table[s, position / block_size] (needle/layers/attention.py:140-154
// for decode, :204-246 for prefill).  nb_slot_mapping resolves that once per
// forward into slots[t] = block * block_size + offset (-1: not written), and
// the writers below take slots[t] with one load instead of walking
// cu_seqlens -> context_lens -> block_table in every layer's launch.
//
// The writers give one warp a (token, group of vectors) unit: the token's
// slot is one broadcast load that overlaps the source loads, there is no
// shared memory and no block-wide barrier, and consecutive lanes move
// consecutive 16-byte vectors of one head row (coalesced reads of the
// token-major K/V rows and of the 256-byte cache rows they land in).
#pragma once
#include <algorithm>
#include <cstdlib>
#include <type_traits>

#include "nb_common.cuh"

namespace nb {

// Decode form (one token per sequence): one thread per sequence.
__global__ void __launch_bounds__(256)
    slot_mapping_decode_kernel(const int32_t* __restrict__ bt, int64_t bt_stride, int maxb,
                               const int32_t* __restrict__ ctx, int num_seqs, int block_size,
                               int num_blocks, int32_t* __restrict__ slots) {
  griddep_launch_dependents();
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= num_seqs) return;
  int phys = -1, off = 0;
  // slot_of restates needle's index math, clamp and last-token-wins rule
  const bool ok =
      slot_of(s, 0, 1, __ldg(ctx + s), bt, bt_stride, maxb, num_blocks, block_size, phys, off);
  slots[s] = ok ? phys * block_size + off : -1;
}

// Prefill form: CTAs stride over sequences, a sequence's tokens over threads,
// so a token costs its sequence's two bounds and one table entry (no search).
__global__ void __launch_bounds__(256)
    slot_mapping_prefill_kernel(const int32_t* __restrict__ bt, int64_t bt_stride, int maxb,
                                const int32_t* __restrict__ cu, const int32_t* __restrict__ ctx,
                                int num_seqs, int block_size, int num_blocks,
                                int32_t* __restrict__ slots) {
  griddep_launch_dependents();
  for (int s = blockIdx.x; s < num_seqs; s += gridDim.x) {
    const int c0 = __ldg(cu + s), len = __ldg(cu + s + 1) - c0, c = __ldg(ctx + s);
    for (int i = threadIdx.x; i < len; i += blockDim.x) {
      int phys = -1, off = 0;
      const bool ok =
          slot_of(s, i, len, c, bt, bt_stride, maxb, num_blocks, block_size, phys, off);
      slots[c0 + i] = ok ? phys * block_size + off : -1;
    }
  }
}

// Element offset of head 0's row of `slot` in the K half (the V half is
// `half` elements further; head h is h * block_size * D further).  Returns -1
// for a slot that is not written or lies outside the pool (recorded).
__device__ __forceinline__ int64_t slot_base(int slot, int num_blocks, int kvh, int block_size,
                                             int D) {
  if (slot < 0) return -1;
  const int phys = slot / block_size;
  if (phys >= num_blocks) {
    set_error(kErrBlockId);
    return -1;
  }
  const int off = slot - phys * block_size;
  return ((int64_t)phys * kvh * block_size + off) * D;
}

// K/V rows into the cache.  Unit = (token, U x 32 vectors of the token's
// kvh x 2 x vpr vectors, ordered (head, K/V, vector)); warps grid-stride over
// units (host-checked to fit int32).  VPR: vectors per head row when known at
// compile time (0: runtime).
template <typename T, int VPR, int U>
__global__ void __launch_bounds__(256)
    store_kvcache_slots_kernel(const T* __restrict__ k, int64_t k_stride, const T* __restrict__ v,
                               int64_t v_stride, T* __restrict__ cache, int num_blocks, int kvh,
                               int block_size, int D, const int32_t* __restrict__ slots,
                               int num_tokens) {
  // launched with programmatic stream serialisation: the launch overlaps the
  // previous kernel's tail, the reads wait for its results
  griddep_wait();
  griddep_launch_dependents();  // the paged decode that follows may start its launch
  constexpr int VEC = 16 / sizeof(T);
  const int vpr = VPR ? VPR : D / VEC;
  const int per_tok = kvh * 2 * vpr;
  const int upt = (per_tok + 32 * U - 1) / (32 * U);  // units per token
  const int units = num_tokens * upt;
  const int lane = threadIdx.x & 31;
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  const int64_t half = (int64_t)num_blocks * kvh * block_size * D;
  const int64_t head = (int64_t)block_size * D;
  // load(w): the unit's slot and source vectors; store(w): the vectors into
  // the cache.  A warp's next unit is loaded before the current one is
  // stored, so each warp keeps two units of reads in flight.
  auto load = [&](int w, uint4 (&val)[U], int& t, int& slot) {
    t = w / upt;
    const int j0 = (w - t * upt) * 32 * U;
    slot = __ldg(slots + t);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = j0 + u * 32 + lane;
      if (j < per_tok) {
        const int vec = j % vpr, r = j / vpr;
        const T* src = ((r & 1) ? v + (int64_t)t * v_stride : k + (int64_t)t * k_stride) +
                       (int64_t)(r >> 1) * D + vec * VEC;
        val[u] = __ldg(reinterpret_cast<const uint4*>(src));
      }
    }
  };
  auto store = [&](int w, const uint4 (&val)[U], int t, int slot) {
    const int j0 = (w - t * upt) * 32 * U;
    const int64_t base = slot_base(slot, num_blocks, kvh, block_size, D);
    if (base < 0) return;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = j0 + u * 32 + lane;
      if (j < per_tok) {
        const int vec = j % vpr, r = j / vpr;
        T* dst = cache + base + ((r & 1) ? half : 0) + (r >> 1) * head + vec * VEC;
        *reinterpret_cast<uint4*>(dst) = val[u];
      }
    }
  };
  int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (w >= units) return;
  uint4 cur[U];
  int t = 0, slot = -1;
  load(w, cur, t, slot);
  while (true) {
    const int wn = w + nwarps;
    uint4 nxt[U];
    int tn = 0, sn = -1;
    if (wn < units) load(wn, nxt, tn, sn);
    store(w, cur, t, slot);
    if (wn >= units) break;
    w = wn;
    t = tn;
    slot = sn;
#pragma unroll
    for (int u = 0; u < U; ++u) cur[u] = nxt[u];
  }
}

// RoPE of q (in place) and k, then K/V into the cache.  Unit = (token, U x 32
// chunks of the token's (hq + 2 hk) x cpr chunks, ordered (head slot, chunk));
// head slots [0, hq) are q, [hq, hq+hk) k, [hq+hk, hq+2hk) v; a chunk is VEC
// element pairs (x[j..j+VEC), x[j+D/2..j+D/2+VEC)).  Rounding as rope_pair.
template <typename T, int CPR, int U>
__global__ void __launch_bounds__(256)
    rope_store_slots_kernel(T* q, int64_t q_stride, int hq, T* k, int64_t k_stride,
                            const T* __restrict__ v, int64_t v_stride, const T* __restrict__ cos,
                            const T* __restrict__ sin, int64_t cs_stride, T* __restrict__ cache,
                            int num_blocks, int hk, int block_size, int D,
                            const int32_t* __restrict__ slots, int num_tokens,
                            int write_k_back) {
  griddep_wait();  // programmatic launch, as store_kvcache_slots_kernel
  griddep_launch_dependents();
  constexpr int VEC = 16 / sizeof(T);
  const int half = D / 2;
  const int cpr = CPR ? CPR : half / VEC;
  const int per_tok = (hq + 2 * hk) * cpr;
  const int upt = (per_tok + 32 * U - 1) / (32 * U);
  const int units = num_tokens * upt;
  const int lane = threadIdx.x & 31;
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  const int64_t half_cache = (int64_t)num_blocks * hk * block_size * D;
  const int64_t head = (int64_t)block_size * D;
  for (int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < units; w += nwarps) {
    const int t = w / upt;
    const int j0 = (w - t * upt) * 32 * U;
    const int slot = __ldg(slots + t);
    const T* cs = cos + (int64_t)t * cs_stride;
    const T* sn = sin + (int64_t)t * cs_stride;
    // With cpr dividing 32 a lane's chunk column is the same for every head it
    // touches, so its cos/sin chunks load once per unit, alongside the rows.
    constexpr bool kOneCs = CPR != 0 && 32 % (CPR ? CPR : 1) == 0;
    T lo[U][VEC], hi[U][VEC], cl[VEC], ch[VEC], sl[VEC], sh[VEC];
    auto load_cs = [&](int c) {
      *reinterpret_cast<uint4*>(cl) = __ldg(reinterpret_cast<const uint4*>(cs + c));
      *reinterpret_cast<uint4*>(ch) = __ldg(reinterpret_cast<const uint4*>(cs + c + half));
      *reinterpret_cast<uint4*>(sl) = __ldg(reinterpret_cast<const uint4*>(sn + c));
      *reinterpret_cast<uint4*>(sh) = __ldg(reinterpret_cast<const uint4*>(sn + c + half));
    };
    if constexpr (kOneCs) load_cs((lane % cpr) * VEC);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = j0 + u * 32 + lane;
      if (j >= per_tok) continue;
      const int hh = j / cpr, c = (j - hh * cpr) * VEC;
      const T* row = hh < hq        ? q + (int64_t)t * q_stride + (int64_t)hh * D
                     : hh < hq + hk ? k + (int64_t)t * k_stride + (int64_t)(hh - hq) * D
                                    : v + (int64_t)t * v_stride + (int64_t)(hh - hq - hk) * D;
      *reinterpret_cast<uint4*>(lo[u]) = *reinterpret_cast<const uint4*>(row + c);
      *reinterpret_cast<uint4*>(hi[u]) = *reinterpret_cast<const uint4*>(row + c + half);
    }
    const int64_t base = slot_base(slot, num_blocks, hk, block_size, D);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = j0 + u * 32 + lane;
      if (j >= per_tok) continue;
      const int hh = j / cpr, c = (j - hh * cpr) * VEC;
      if (hh < hq + hk) {  // rotate q and k
        if constexpr (!kOneCs) load_cs(c);
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          float ol, oh;
          rope_pair<T>(Dt<T>::to_f(lo[u][e]), Dt<T>::to_f(hi[u][e]), Dt<T>::to_f(cl[e]),
                       Dt<T>::to_f(ch[e]), Dt<T>::to_f(sl[e]), Dt<T>::to_f(sh[e]), ol, oh);
          lo[u][e] = Dt<T>::from_f(ol);
          hi[u][e] = Dt<T>::from_f(oh);
        }
        if (hh < hq || write_k_back) {
          T* row = hh < hq ? q + (int64_t)t * q_stride + (int64_t)hh * D
                           : k + (int64_t)t * k_stride + (int64_t)(hh - hq) * D;
          *reinterpret_cast<uint4*>(row + c) = *reinterpret_cast<uint4*>(lo[u]);
          *reinterpret_cast<uint4*>(row + c + half) = *reinterpret_cast<uint4*>(hi[u]);
        }
      }
      if (hh >= hq && base >= 0) {  // k and v rows into the cache
        const bool is_k = hh < hq + hk;
        const int h = is_k ? hh - hq : hh - hq - hk;
        T* dst = cache + base + (is_k ? 0 : half_cache) + h * head + c;
        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<uint4*>(lo[u]);
        *reinterpret_cast<uint4*>(dst + half) = *reinterpret_cast<uint4*>(hi[u]);
      }
    }
  }
}

}  // namespace nb

namespace nbh {

// Warps for `units` work units: enough CTAs of 8 warps for one unit per warp,
// capped at a few resident waves (the kernels grid-stride; NB_KVW_WAVES=1..4
// sets the cap, diagnostics).
inline unsigned slot_grid(int64_t units) {
  static int waves = [] {
    const char* e = getenv("NB_KVW_WAVES");
    return (e && e[0] >= '1' && e[0] <= '4') ? e[0] - '0' : 4;
  }();
  const int64_t cap = (int64_t)num_sms() * 8 * waves;
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>((units + 7) / 8, cap));
}

inline bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

// 16-byte vectors per lane and unit of the slot writers: 2, 4 or 8
// (NB_KVW_U, diagnostics).
inline int kvw_unroll() {
  static int v = [] {
    const char* e = getenv("NB_KVW_U");
    return (e && e[0] == '8') ? 8 : (e && e[0] == '2') ? 2 : 4;
  }();
  return v;
}

template <typename T>
int launch_store_slots(const void* k, int64_t ks, const void* v, int64_t vs, void* cache,
                       int nblk, int kvh, int bs, int D, const int32_t* slots, int ntok,
                       cudaStream_t st) {
  constexpr int VEC = 16 / sizeof(T);
  if (D % VEC || ks % VEC || vs % VEC || !aligned16(k) || !aligned16(v) || !aligned16(cache))
    return fail(NB_ERR_UNSUPPORTED,
                "slot writers need 16-byte aligned rows (head_dim and strides multiples of %d)",
                VEC);
  const int per_tok = kvh * 2 * (D / VEC);
  auto go = [&](auto u_tag) -> int {
    constexpr int U = decltype(u_tag)::value;
    const int64_t units = (int64_t)ntok * ((per_tok + 32 * U - 1) / (32 * U));
    if (units > INT32_MAX / 2) return fail(NB_ERR_UNSUPPORTED, "too many tokens for one launch");
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr[1];
    pdl_config(cfg, attr, dim3(slot_grid(units)), dim3(256), 0, st);
    auto kern = D / VEC == 16  ? nb::store_kvcache_slots_kernel<T, 16, U>
                : D / VEC == 8 ? nb::store_kvcache_slots_kernel<T, 8, U>
                               : nb::store_kvcache_slots_kernel<T, 0, U>;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, (const T*)k, ks, (const T*)v, vs, (T*)cache,
                                       nblk, kvh, bs, D, slots, ntok);
    if (e != cudaSuccess)
      return fail(NB_ERR_CUDA, "store_kvcache_slots launch: %s", cudaGetErrorString(e));
    return check_launch("store_kvcache_slots");
  };
  if (kvw_unroll() == 8) return go(std::integral_constant<int, 8>());
  if (kvw_unroll() == 2) return go(std::integral_constant<int, 2>());
  return go(std::integral_constant<int, 4>());
}

template <typename T>
int launch_rope_store_slots(void* q, int64_t qs, int hq, void* k, int64_t ks, const void* v,
                            int64_t vs, const void* cos, const void* sin, int64_t css,
                            void* cache, int nblk, int hk, int bs, int D, const int32_t* slots,
                            int ntok, int wkb, cudaStream_t st) {
  constexpr int VEC = 16 / sizeof(T);
  if ((D / 2) % VEC || qs % VEC || ks % VEC || vs % VEC || css % VEC || !aligned16(q) ||
      !aligned16(k) || !aligned16(v) || !aligned16(cos) || !aligned16(sin) || !aligned16(cache))
    return fail(NB_ERR_UNSUPPORTED,
                "slot writers need 16-byte aligned rows (head_dim / 2 and strides multiples of "
                "%d)", VEC);
  constexpr int U = 2;
  const int cpr = D / 2 / VEC;
  const int per_tok = (hq + 2 * hk) * cpr;
  const int64_t units = (int64_t)ntok * ((per_tok + 32 * U - 1) / (32 * U));
  if (units > INT32_MAX / 2) return fail(NB_ERR_UNSUPPORTED, "too many tokens for one launch");
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute attr[1];
  pdl_config(cfg, attr, dim3(slot_grid(units)), dim3(256), 0, st);
  auto kern = cpr == 8   ? nb::rope_store_slots_kernel<T, 8, U>
              : cpr == 4 ? nb::rope_store_slots_kernel<T, 4, U>
                         : nb::rope_store_slots_kernel<T, 0, U>;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, (T*)q, qs, hq, (T*)k, ks, (const T*)v, vs,
                                     (const T*)cos, (const T*)sin, css, (T*)cache, nblk, hk, bs,
                                     D, slots, ntok, wkb);
  if (e != cudaSuccess)
    return fail(NB_ERR_CUDA, "rope_store_kvcache_slots launch: %s", cudaGetErrorString(e));
  return check_launch("rope_store_kvcache_slots");
}

inline int check_slot_cache(const void* cache, int nblk, int kvh, int bs, int D,
                            const int32_t* slots, int ntok) {
  if (!cache || !slots) return fail(NB_ERR_INVALID_ARG, "null cache/slots");
  if (nblk <= 0 || kvh <= 0 || bs <= 0 || D <= 0 || ntok < 0)
    return fail(NB_ERR_INVALID_ARG, "non-positive cache dimension or negative token count");
  if ((int64_t)nblk * bs > INT32_MAX)
    return fail(NB_ERR_UNSUPPORTED, "num_blocks * block_size exceeds int32 slots");
  return NB_OK;
}

}  // namespace nbh

extern "C" {

int nb_slot_mapping(const int32_t* block_table, int64_t block_table_stride,
                    int max_blocks_per_seq, const int32_t* cu_seqlens,
                    const int32_t* context_lens, int num_seqs, int num_tokens, int block_size,
                    int num_blocks, int32_t* slots, void* stream) {
  using namespace nbh;
  if (!block_table || !context_lens || !slots)
    return fail(NB_ERR_INVALID_ARG, "null block_table/context_lens/slots");
  if (num_seqs < 0 || num_tokens < 0 || block_size <= 0 || num_blocks <= 0 ||
      max_blocks_per_seq <= 0)
    return fail(NB_ERR_INVALID_ARG, "bad sizes");
  if (block_table_stride < max_blocks_per_seq)
    return fail(NB_ERR_INVALID_ARG, "block_table_stride < max_blocks_per_seq");
  if ((int64_t)num_blocks * block_size > INT32_MAX)
    return fail(NB_ERR_UNSUPPORTED, "num_blocks * block_size exceeds int32 slots");
  if (!cu_seqlens && num_tokens != num_seqs)
    return fail(NB_ERR_INVALID_ARG, "cu_seqlens NULL requires num_tokens == num_seqs");
  if (num_tokens == 0) return NB_OK;
  if (num_seqs == 0) return fail(NB_ERR_INVALID_ARG, "tokens without sequences");
  cudaStream_t st = (cudaStream_t)stream;
  if (!cu_seqlens)
    nb::slot_mapping_decode_kernel<<<(num_seqs + 255) / 256, 256, 0, st>>>(
        block_table, block_table_stride, max_blocks_per_seq, context_lens, num_seqs, block_size,
        num_blocks, slots);
  else
    nb::slot_mapping_prefill_kernel<<<std::min(num_seqs, num_sms() * 8), 256, 0, st>>>(
        block_table, block_table_stride, max_blocks_per_seq, cu_seqlens, context_lens, num_seqs,
        block_size, num_blocks, slots);
  return check_launch("slot_mapping");
}

int nb_store_kvcache_slots(const void* k, int64_t k_stride, const void* v, int64_t v_stride,
                           void* kv_cache, int num_blocks, int num_kv_heads, int block_size,
                           int head_dim, const int32_t* slots, int num_tokens, int dtype,
                           void* stream) {
  using namespace nbh;
  if (!valid_dtype(dtype)) return fail(NB_ERR_INVALID_ARG, "invalid dtype %d", dtype);
  if (int rc = check_slot_cache(kv_cache, num_blocks, num_kv_heads, block_size, head_dim, slots,
                                num_tokens))
    return rc;
  if (!k || !v) return fail(NB_ERR_INVALID_ARG, "null k/v");
  if (k_stride < (int64_t)num_kv_heads * head_dim || v_stride < (int64_t)num_kv_heads * head_dim)
    return fail(NB_ERR_INVALID_ARG, "k/v row stride smaller than num_kv_heads * head_dim");
  if (num_tokens == 0) return NB_OK;
  cudaStream_t st = (cudaStream_t)stream;
  switch (dtype) {
    case NB_DTYPE_F32:
      return launch_store_slots<float>(k, k_stride, v, v_stride, kv_cache, num_blocks,
                                       num_kv_heads, block_size, head_dim, slots, num_tokens, st);
    case NB_DTYPE_F16:
      return launch_store_slots<__half>(k, k_stride, v, v_stride, kv_cache, num_blocks,
                                        num_kv_heads, block_size, head_dim, slots, num_tokens,
                                        st);
    default:
      return launch_store_slots<__nv_bfloat16>(k, k_stride, v, v_stride, kv_cache, num_blocks,
                                               num_kv_heads, block_size, head_dim, slots,
                                               num_tokens, st);
  }
}

int nb_rope_store_kvcache_slots(void* q, int64_t q_stride, int num_q_heads, void* k,
                                int64_t k_stride, const void* v, int64_t v_stride,
                                const void* cos, const void* sin, int64_t cs_stride,
                                void* kv_cache, int num_blocks, int num_kv_heads, int block_size,
                                int head_dim, const int32_t* slots, int num_tokens,
                                int write_k_back, int dtype, void* stream) {
  using namespace nbh;
  if (!valid_dtype(dtype)) return fail(NB_ERR_INVALID_ARG, "invalid dtype %d", dtype);
  if (int rc = check_slot_cache(kv_cache, num_blocks, num_kv_heads, block_size, head_dim, slots,
                                num_tokens))
    return rc;
  if (!q || !k || !v || !cos || !sin) return fail(NB_ERR_INVALID_ARG, "null q/k/v/cos/sin");
  if (head_dim % 2) return fail(NB_ERR_INVALID_ARG, "head_dim must be even");
  if (num_q_heads <= 0) return fail(NB_ERR_INVALID_ARG, "num_q_heads must be > 0");
  if (q_stride < (int64_t)num_q_heads * head_dim ||
      k_stride < (int64_t)num_kv_heads * head_dim ||
      v_stride < (int64_t)num_kv_heads * head_dim || cs_stride < head_dim)
    return fail(NB_ERR_INVALID_ARG, "row stride too small");
  if (num_tokens == 0) return NB_OK;
  cudaStream_t st = (cudaStream_t)stream;
  switch (dtype) {
    case NB_DTYPE_F32:
      return launch_rope_store_slots<float>(q, q_stride, num_q_heads, k, k_stride, v, v_stride,
                                            cos, sin, cs_stride, kv_cache, num_blocks,
                                            num_kv_heads, block_size, head_dim, slots,
                                            num_tokens, write_k_back, st);
    case NB_DTYPE_F16:
      return launch_rope_store_slots<__half>(q, q_stride, num_q_heads, k, k_stride, v, v_stride,
                                             cos, sin, cs_stride, kv_cache, num_blocks,
                                             num_kv_heads, block_size, head_dim, slots,
                                             num_tokens, write_k_back, st);
    default:
      return launch_rope_store_slots<__nv_bfloat16>(
          q, q_stride, num_q_heads, k, k_stride, v, v_stride, cos, sin, cs_stride, kv_cache,
          num_blocks, num_kv_heads, block_size, head_dim, slots, num_tokens, write_k_back, st);
  }
}

}  // extern "C"
