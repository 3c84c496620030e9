// Tensor-parallel all-reduce fused with the residual add and RMSNorm.
//
// Under TP the row-parallel o_proj / down_proj leave a partial [T, hidden]
// sum on every rank (needle/layers/linear.py:92-98 all-reduces it with NCCL)
// and the decoder then adds the residual and normalises
// (needle/model/llama.py:67-72).  This kernel does all three in one launch
// over NVLink peer memory, as a reduce-scatter followed by an all-gather,
// with no flag words: the data is its own arrival signal.
//
//   * Every receive buffer starts filled with a sentinel bit pattern (0xFFFF
//     in every 16-bit lane, a NaN) that valid data never holds: senders
//     rewrite that one NaN pattern to another NaN (0x7FFF) before storing.
//     A reader polls a 16-byte vector until none of its lanes is the
//     sentinel, consumes it, and later writes the sentinel back.
//   * Rank q owns rows [q*R, q*R+R) (R = ceil(T / world)).  CTA b of every
//     rank handles row index b: it pushes its partial of row q*R+b into
//     owner q's receive slot [sender][b]; as owner it waits for all world
//     slots of its row b, sums them in rank order 0..W-1 (the same order on
//     every owner: identical bits everywhere), rounds to the storage type
//     (the all-reduced tensor), adds the residual, normalises, and pushes
//     the new residual row and the normalised row into every rank's gather
//     slot [owner][b]; finally it waits for the world gather slots of index
//     b and copies them into this rank's residual and output rows.
//   * When the GPU holds two CTAs per row index at once, the second
//     receives the gathered normalised rows while the first receives the
//     residual rows, so both receive batches are in flight together.
//   * Receive and gather buffers are double-buffered by the parity of a
//     per-row-index call counter (epochs[role][b]; a call without the second
//     role advances both counters, so they never drift apart).  A sender writes a buffer half
//     again two calls later; by then its previous call has received this
//     rank's results of the call in between, which this rank sent after it
//     had consumed (and reset) the half being rewritten.
//
// Memory ordering.  Every access another GPU can observe is strong
// (ld.relaxed.sys polls, st.relaxed.sys pushes and sentinel resets), and the
// data is its own arrival signal per 16-bit lane, so no data word needs to be
// ordered before another.  The one hazard is a late sentinel reset: rank A
// resets slot X (in its own memory) after consuming it, and sender B writes X
// again two calls later; the reset must not land after B's new data.  A
// thread resets its consumed slots only after it has issued all of its pushes
// of the call, so B's next write to X is causally after a push that A makes
// in a LATER launch (B's call two steps on waits, directly or through rank 0's
// gather that every rank receives, for data that A pushed in the call in
// between).  Launches on one stream are ordered: A's later launch starts
// only after every store of the earlier one has been performed at A's L2,
// which is also where B's NVLink store to X lands (the point of coherence of
// A's memory).  So B's write is ordered after A's reset in X's coherence
// order, without any fence in the kernel; a reader never acts on a slot
// before its own poll returned the data (no speculative stores).
//
// Failure: every wait is bounded (nb_tp_set_wait_limit_ns, 2 s by default).
// A CTA that gives up records NB_DEVERR_TIMEOUT, sets the communicator's
// status word (device memory, epochs[kArStatusWord]) and, when given, a
// host-visible word in pinned memory, and returns.  The slots are then in an
// unknown state, so every later call that finds the status word set returns
// at once without touching them: the communicator stays poisoned until the
// host refills the buffers with the sentinel and zeroes the counters and the
// status word on every rank (TPComm.reset()).
#pragma once
#include <algorithm>
#include <atomic>
#include <cstring>

#include "nb_common.cuh"

namespace nb {

constexpr int kArMaxRanks = 8;
constexpr int kArMaxRows = 1024;  // rows per rank (row indices b); epochs hold 2 x this
constexpr int kArStatusWord = 2 * kArMaxRows;  // epochs[kArStatusWord]: non-zero = poisoned
constexpr int kArEpochWords = 2 * kArMaxRows + 32;
static_assert(kArEpochWords == NB_TP_EPOCH_WORDS && kArStatusWord == NB_TP_STATUS_WORD,
              "the header's epoch layout");

struct ArPeers {
  void* recv[kArMaxRanks];    // each rank's receive slots [2][world][slot_rows][hidden]
  void* gather[kArMaxRanks];  // each rank's gather slots [2][world][slot_rows][2][hidden]
};

constexpr unsigned kArSentinel = 0xFFFFFFFFu;

__device__ __forceinline__ uint4 ld_relaxed_sys_v4(const void* p) {
  uint4 v;
  asm volatile("ld.relaxed.sys.global.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_sys_v4(void* p, const uint4& v) {
  asm volatile("st.relaxed.sys.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ bool lane_is_sentinel(unsigned w) {
  return (w & 0xFFFFu) == 0xFFFFu || (w >> 16) == 0xFFFFu;
}
__device__ __forceinline__ bool arrived(const uint4& v) {
  return !(lane_is_sentinel(v.x) || lane_is_sentinel(v.y) || lane_is_sentinel(v.z) ||
           lane_is_sentinel(v.w));
}
// The sentinel NaN becomes another NaN, so data never reads as "not arrived".
__device__ __forceinline__ unsigned canon_word(unsigned w) {
  if ((w & 0xFFFFu) == 0xFFFFu) w = (w & 0xFFFF0000u) | 0x7FFFu;
  if ((w >> 16) == 0xFFFFu) w = (w & 0x0000FFFFu) | 0x7FFF0000u;
  return w;
}
__device__ __forceinline__ uint4 canon(uint4 v) {
  return make_uint4(canon_word(v.x), canon_word(v.y), canon_word(v.z), canon_word(v.w));
}

// N vectors at base + i * stride (elements of 16-bit T), i < n: all loads in
// flight at once; while some have not arrived, all of the missing ones are
// loaded again together, so every pass costs one memory round trip however
// many senders are late.  Gives up (dead = true) after wait_ns, or at once if
// an earlier wait of this thread already gave up.
template <int N, typename T>
__device__ __forceinline__ void poll_vecs(const T* base, int64_t stride, int n, uint4 (&v)[N],
                                          bool& dead, unsigned long long wait_ns) {
  unsigned missing = 0;
#pragma unroll
  for (int i = 0; i < N; ++i)
    if (i < n) v[i] = ld_relaxed_sys_v4(base + i * stride);
#pragma unroll
  for (int i = 0; i < N; ++i)
    if (i < n && !arrived(v[i])) missing |= 1u << i;
  if (missing && !dead) {
    const unsigned long long t0 = globaltimer();
    while (missing) {
#pragma unroll
      for (int i = 0; i < N; ++i)
        if (missing & (1u << i)) v[i] = ld_relaxed_sys_v4(base + i * stride);
#pragma unroll
      for (int i = 0; i < N; ++i)
        if ((missing & (1u << i)) && arrived(v[i])) missing &= ~(1u << i);
      if (missing && globaltimer() - t0 > wait_ns) {
        dead = true;
        break;
      }
    }
  }
}

// Write the sentinel back into n consumed slots (strong stores: a peer's next
// write to the slot must come after them in the slot's coherence order).
template <int N, typename T>
__device__ __forceinline__ void reset_vecs(T* base, int64_t stride, int n) {
  const uint4 sentinel = make_uint4(kArSentinel, kArSentinel, kArSentinel, kArSentinel);
#pragma unroll
  for (int i = 0; i < N; ++i)
    if (i < n) st_relaxed_sys_v4(base + i * stride, sentinel);
}

template <typename T, int VEC, int MAXW>
__global__ void __launch_bounds__(1024)
    tp_allreduce_add_rmsnorm_kernel(const __grid_constant__ ArPeers P, const T* __restrict__ partial,
                                    T* __restrict__ out, T* __restrict__ res, int slot_rows,
                                    unsigned* __restrict__ epochs, unsigned* host_status,
                                    int rank, int world, const T* __restrict__ weight, int rows,
                                    int hidden, float eps, int split,
                                    unsigned long long wait_ns) {
  static_assert(VEC * sizeof(T) == 16, "one 16-byte vector per thread");
  static_assert(MAXW <= kArMaxRanks, "rank capacity");
  __shared__ float red[32];
  __shared__ unsigned s_e, s_poison;
  const int per = (rows + world - 1) / world;
  const int nvec = hidden / VEC;
  const bool mine = threadIdx.x < nvec;  // one vector per thread (hidden <= 1024 * VEC)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t col = (int64_t)threadIdx.x * VEC;
  const int64_t slot = (int64_t)slot_rows * hidden;  // elements per sender slot
  // With split, two CTAs per row index b: role 0 pushes, reduces the rows it
  // owns and receives the gathered residual rows; role 1 receives the
  // gathered normalised rows, so that both receive batches are in flight
  // together.  Without split (more row indices than resident CTA pairs),
  // role 0 receives both.
  const int G = split ? gridDim.x >> 1 : gridDim.x;
  const int role = split && blockIdx.x >= G;
  unsigned* ep = epochs + role * kArMaxRows;  // per-role call counters
  volatile unsigned* status = epochs + kArStatusWord;
  bool dead = false;
  uint4 v[MAXW];
  // The grid is at most what fits on the GPU at once (every CTA resident), so
  // a CTA waiting on a peer never blocks the CTA that the peer waits for.
  for (int b = blockIdx.x - role * G; b < per; b += G) {
    if (threadIdx.x == 0) {
      s_e = ep[b];
      s_poison = *status;
    }
    // owners q with a row at index b: q*per+b < rows
    const int nq = min(world, (rows - 1 - b) / per + 1);
    if (role == 0) {
      // 1. reduce-scatter: row q*per+b of this rank's partial -> owner q, slot [rank][b]
      //    (the partial loads overlap the call-counter load)
      if (mine) {
#pragma unroll
        for (int q = 0; q < MAXW; ++q)
          if (q < nq)
            v[q] = *reinterpret_cast<const uint4*>(partial + (int64_t)(q * per + b) * hidden + col);
      }
      __syncthreads();
      if (s_poison) return;  // poisoned by an earlier timeout: touch nothing
      const int par = s_e & 1;
      if (mine) {
#pragma unroll
        for (int q = 0; q < MAXW; ++q)
          if (q < nq)
            st_relaxed_sys_v4(reinterpret_cast<T*>(P.recv[q]) +
                                  ((int64_t)par * world + rank) * slot + (int64_t)b * hidden + col,
                              canon(v[q]));
      }
      // 2. owner of row rank*per+b: sum the world slots, residual, RMSNorm, all-gather
      const int row = rank * per + b;
      if (row < rows) {  // uniform over the CTA
        float ss = 0.f;
        T hv[VEC];
        T* rb = reinterpret_cast<T*>(P.recv[rank]) + (int64_t)par * world * slot +
                (int64_t)b * hidden + col;
        if (mine) {
          T rv[VEC];
          *reinterpret_cast<uint4*>(rv) =
              *reinterpret_cast<const uint4*>(res + (int64_t)row * hidden + col);
          poll_vecs<MAXW>(rb, slot, world, v, dead, wait_ns);
          float acc[VEC];
#pragma unroll
          for (int k = 0; k < VEC; ++k) acc[k] = 0.f;
#pragma unroll
          for (int p = 0; p < MAXW; ++p) {  // fixed rank order: identical bits everywhere
            if (p < world) {
              const T* x = reinterpret_cast<const T*>(&v[p]);
#pragma unroll
              for (int k = 0; k < VEC; ++k) acc[k] = __fadd_rn(acc[k], Dt<T>::to_f(x[k]));
            }
          }
#pragma unroll
          for (int k = 0; k < VEC; ++k) {
            // all-reduced value rounded to the storage type, then residual + it
            const float sum = Dt<T>::round(acc[k]);
            hv[k] = Dt<T>::from_f(__fadd_rn(Dt<T>::to_f(rv[k]), sum));
            const float f = Dt<T>::to_f(hv[k]);
            ss = __fadd_rn(ss, __fmul_rn(f, f));
          }
        }
        // the weight load's latency hides behind the block reduction
        uint4 w4 = make_uint4(0, 0, 0, 0);
        if (mine) w4 = __ldg(reinterpret_cast<const uint4*>(weight + col));
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        if (warp == 0) {
          float x = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
          x = warp_sum(x);
          if (lane == 0) red[0] = x;
        }
        __syncthreads();
        if (mine) {
          const float var = __fdiv_rn(red[0], (float)hidden);
          const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
          const T* wv = reinterpret_cast<const T*>(&w4);
          T ov[VEC];
#pragma unroll
          for (int k = 0; k < VEC; ++k) {
            const float xn = Dt<T>::round(__fmul_rn(Dt<T>::to_f(hv[k]), r));
            ov[k] = Dt<T>::from_f(__fmul_rn(Dt<T>::to_f(wv[k]), xn));
          }
          const uint4 h4 = canon(*reinterpret_cast<uint4*>(hv));
          const uint4 o4 = canon(*reinterpret_cast<uint4*>(ov));
          const int64_t g =
              ((int64_t)par * world + rank) * 2 * slot + (int64_t)b * 2 * hidden + col;
          // A thread whose wait ran out pushes nothing more, so every rank
          // that needs its rows times out as well instead of reading garbage.
          if (!dead) {
#pragma unroll
            for (int p = 0; p < MAXW; ++p) {
              if (p < world) {
                T* gp = reinterpret_cast<T*>(P.gather[p]) + g;
                st_relaxed_sys_v4(gp, h4);
                st_relaxed_sys_v4(gp + hidden, o4);
              }
            }
            // the consumed receive slots, reset after this call's pushes (they
            // are written again two calls later, after a later launch)
            reset_vecs<MAXW>(rb, slot, world);
          }
        }
      }
      // 3. all-gather receive, residual rows q*per+b from their owners q
      if (mine && !dead) {
        T* gb = reinterpret_cast<T*>(P.gather[rank]) + (int64_t)par * world * 2 * slot +
                (int64_t)b * 2 * hidden + col;
        poll_vecs<MAXW>(gb, 2 * slot, nq, v, dead, wait_ns);
        if (!dead) {
#pragma unroll
          for (int q = 0; q < MAXW; ++q)
            if (q < nq)
              *reinterpret_cast<uint4*>(res + (int64_t)(q * per + b) * hidden + col) = v[q];
          reset_vecs<MAXW>(gb, 2 * slot, nq);
        }
        if (!split && !dead) {
          poll_vecs<MAXW>(gb + hidden, 2 * slot, nq, v, dead, wait_ns);
          if (!dead) {
#pragma unroll
            for (int q = 0; q < MAXW; ++q)
              if (q < nq)
                *reinterpret_cast<uint4*>(out + (int64_t)(q * per + b) * hidden + col) = v[q];
            reset_vecs<MAXW>(gb + hidden, 2 * slot, nq);
          }
        }
      }
    } else {
      __syncthreads();
      if (s_poison) return;
      const int par = s_e & 1;
      // 3'. all-gather receive, normalised rows q*per+b from their owners q
      if (mine) {
        T* gb = reinterpret_cast<T*>(P.gather[rank]) + (int64_t)par * world * 2 * slot +
                (int64_t)b * 2 * hidden + hidden + col;
        poll_vecs<MAXW>(gb, 2 * slot, nq, v, dead, wait_ns);
        if (!dead) {
#pragma unroll
          for (int q = 0; q < MAXW; ++q)
            if (q < nq)
              *reinterpret_cast<uint4*>(out + (int64_t)(q * per + b) * hidden + col) = v[q];
          reset_vecs<MAXW>(gb, 2 * slot, nq);
        }
      }
    }
    if (__syncthreads_or(dead)) {
      if (threadIdx.x == 0) {
        set_error(kErrTimeout);
        *status = 1u;
        if (host_status) *reinterpret_cast<volatile unsigned*>(host_status) = 1u;
        __threadfence_system();
      }
      return;
    }
    if (threadIdx.x == 0) {
      ep[b] = s_e + 1;
      // Without split, role 0 also received the normalised rows: advance the
      // second role's counter too, so both stay in step (the owners chose the
      // gather slot half by role 0's counter) when a later call splits.
      if (!split) epochs[kArMaxRows + b] = s_e + 1;
    }
  }
}

}  // namespace nb

extern "C" {

int nb_ipc_handle(const void* dev_ptr, void* handle_out, uint64_t* offset_out) {
  using namespace nbh;
  if (!dev_ptr || !handle_out || !offset_out) return fail(NB_ERR_INVALID_ARG, "null pointer");
  // The handle names the whole allocation that contains dev_ptr (a caching
  // allocator may have carved dev_ptr out of a larger one): report the offset.
  static PFN_cuMemGetAddressRange_v3020 range = nullptr;
  if (!range) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &fn, 12000, cudaEnableDefault,
                                         &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return fail(NB_ERR_CUDA, "cuMemGetAddressRange is not available from the driver");
    range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, (CUdeviceptr)dev_ptr) != CUDA_SUCCESS)
    return fail(NB_ERR_CUDA, "cuMemGetAddressRange failed");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, (void*)base);
  if (e != cudaSuccess) return fail(NB_ERR_CUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = (uint64_t)((CUdeviceptr)dev_ptr - base);
  return NB_OK;
}

int nb_ipc_open(const void* handle, void** dev_ptr_out) {
  using namespace nbh;
  if (!handle || !dev_ptr_out) return fail(NB_ERR_INVALID_ARG, "null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(dev_ptr_out, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess)
    return fail(NB_ERR_CUDA, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  return NB_OK;
}

int nb_ipc_close(void* dev_ptr) {
  using namespace nbh;
  const cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
  if (e != cudaSuccess)
    return fail(NB_ERR_CUDA, "cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
  return NB_OK;
}

namespace {
std::atomic<unsigned long long> g_ar_wait_ns{0};  // 0: nb::kWaitLimitNs
}

int nb_tp_set_wait_limit_ns(uint64_t ns) {
  if (ns > 60ull * 1000000000ull)
    return nbh::fail(NB_ERR_INVALID_ARG, "wait limit above 60 s");
  g_ar_wait_ns.store(ns);
  return NB_OK;
}

int nb_tp_allreduce_add_rmsnorm(const void* partial, void* const* recv, void* const* gather,
                                int slot_rows, void* out, void* residual, unsigned* epochs,
                                unsigned* host_status, int rank, int world, const void* weight,
                                int num_tokens, int hidden, float eps, int dtype, void* stream) {
  using namespace nbh;
  if (!valid_dtype(dtype) || dtype == NB_DTYPE_F32)
    return fail(NB_ERR_UNSUPPORTED, "fused TP all-reduce supports bf16/fp16");
  if (!partial || !recv || !gather || !out || !residual || !epochs || !weight)
    return fail(NB_ERR_INVALID_ARG, "null pointer argument");
  if (world < 1 || world > nb::kArMaxRanks || rank < 0 || rank >= world)
    return fail(NB_ERR_INVALID_ARG, "rank %d / world %d out of range", rank, world);
  if (num_tokens < 0 || hidden <= 0 || hidden % 8 || hidden > 1024 * 8)
    return fail(NB_ERR_UNSUPPORTED, "hidden must be a multiple of 8 up to 8192");
  const int per = (num_tokens + world - 1) / world;
  if (per > nb::kArMaxRows)
    return fail(NB_ERR_UNSUPPORTED, "%d rows per rank exceed %d", per, nb::kArMaxRows);
  if (per > slot_rows)
    return fail(NB_ERR_INVALID_ARG, "%d rows per rank exceed the %d slot rows", per, slot_rows);
  if (num_tokens == 0) return NB_OK;
  if ((uintptr_t)weight % 16 || (uintptr_t)partial % 16 || (uintptr_t)out % 16 ||
      (uintptr_t)residual % 16)
    return fail(NB_ERR_INVALID_ARG, "weight, partial, out and residual must be 16-byte aligned");
  nb::ArPeers P;
  for (int p = 0; p < world; ++p) {
    if (!recv[p] || !gather[p]) return fail(NB_ERR_INVALID_ARG, "rank %d: null buffer", p);
    if ((uintptr_t)recv[p] % 16 || (uintptr_t)gather[p] % 16)
      return fail(NB_ERR_INVALID_ARG, "rank %d: buffers must be 16-byte aligned", p);
    P.recv[p] = recv[p];
    P.gather[p] = gather[p];
  }
  const int threads = std::max(32, ((hidden / 8 + 31) / 32) * 32);
  cudaStream_t st = (cudaStream_t)stream;
  auto launch = [&](auto kern, auto* type_tag) {
    using T = std::remove_pointer_t<decltype(type_tag)>;
    // at most one resident wave: every CTA runs concurrently with its peers
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, threads, 0) != cudaSuccess ||
        occ < 1)
      return fail(NB_ERR_CUDA, "occupancy query failed");
    const int cap = occ * num_sms();
    const int split = 2 * per <= cap;
    const int grid = split ? 2 * per : std::min(per, cap);
    const unsigned long long w = g_ar_wait_ns.load();
    kern<<<grid, threads, 0, st>>>(P, (const T*)partial, (T*)out, (T*)residual, slot_rows, epochs,
                                   host_status, rank, world, (const T*)weight, num_tokens, hidden,
                                   eps, split, w ? w : nb::kWaitLimitNs);
    return check_launch("tp_allreduce_add_rmsnorm");
  };
  // per-thread vector arrays sized for the group: fewer registers below 8 ranks
#define NB_AR_LAUNCH(W)                                                                      \
  if (world <= W) {                                                                          \
    if (dtype == NB_DTYPE_BF16)                                                              \
      return launch(nb::tp_allreduce_add_rmsnorm_kernel<__nv_bfloat16, 8, W>,                \
                    (__nv_bfloat16*)nullptr);                                                \
    return launch(nb::tp_allreduce_add_rmsnorm_kernel<__half, 8, W>, (__half*)nullptr);      \
  }
  NB_AR_LAUNCH(2)
  NB_AR_LAUNCH(4)
  NB_AR_LAUNCH(8)
#undef NB_AR_LAUNCH
  return fail(NB_ERR_INVALID_ARG, "world %d", world);
}

}  // extern "C"
