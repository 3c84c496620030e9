// Tensor-parallel all-reduce fused with the residual add and RMSNorm.
//
// Under TP the row-parallel o_proj / down_proj leave a partial [T, hidden]
// sum on every rank (needle/layers/linear.py:92-98 all-reduces it with NCCL)
// and the decoder then adds the residual and normalises
// (needle/model/llama.py:67-72).  This kernel does all three in one launch
// over NVLink peer memory:
//   * rank r owns rows [r*R, r*R+R) (R = ceil(T / world)); CTA b of every
//     rank handles row r*R + b of its own rank;
//   * barrier 1: CTA b announces to every peer that this rank's partial is
//     complete (its GEMM finished before this kernel started), then waits
//     until every peer's CTA b has done the same;
//   * it sums the row over all ranks' partial buffers in rank order 0..W-1
//     (the same order on every rank, so every rank computes identical
//     bits), rounds the sum to the storage type (the all-reduced tensor),
//     adds the residual, normalises, and stores the new residual row and the
//     normalised row into every rank's buffers (plain peer stores);
//   * barrier 2: CTA b announces its stores are done and waits for every
//     peer's CTA b.  When all CTAs of a rank have passed it, every peer has
//     written its rows into this rank's buffers.
// Flags hold per-CTA epochs that each rank keeps in its own memory and bumps
// on every call, so the same launch can be replayed from a CUDA graph.
// Waits are bounded; on a timeout the kernel records NB_DEVERR_TIMEOUT and
// returns.  Only plain loads and stores cross NVLink.
#pragma once
#include <algorithm>
#include <cstring>

#include "nb_common.cuh"

namespace nb {

constexpr int kArMaxRanks = 8;
constexpr int kArMaxCtas = 1024;  // rows per rank

struct ArPeers {
  const void* part[kArMaxRanks];  // each rank's partial-sum buffer [T, hidden]
  void* out[kArMaxRanks];         // each rank's normalised-output buffer
  void* res[kArMaxRanks];         // each rank's residual buffer (read and updated)
  unsigned* flags[kArMaxRanks];   // each rank's flags [2][kArMaxCtas][kArMaxRanks]
};

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Signal this CTA's arrival to every rank, then wait for every rank's CTA b.
// Returns false if a peer did not arrive within kWaitLimitNs.
__device__ __forceinline__ bool ar_barrier(const ArPeers& P, int which, int b, int rank, int world,
                                           unsigned e) {
  bool ok = true;
  if (threadIdx.x < world) {
    __threadfence_system();
    st_release_sys(P.flags[threadIdx.x] + ((size_t)which * kArMaxCtas + b) * kArMaxRanks + rank, e);
  }
  if (threadIdx.x < world) {
    const unsigned* f =
        P.flags[rank] + ((size_t)which * kArMaxCtas + b) * kArMaxRanks + threadIdx.x;
    if ((int)(ld_acquire_sys(f) - e) < 0) {
      const unsigned long long t0 = globaltimer();
      while ((int)(ld_acquire_sys(f) - e) < 0) {
        if (globaltimer() - t0 > kWaitLimitNs) { ok = false; break; }
      }
    }
  }
  return __syncthreads_and(ok) != 0;
}

template <typename T, int VEC>
__global__ void __launch_bounds__(1024)
    tp_allreduce_add_rmsnorm_kernel(const __grid_constant__ ArPeers P, unsigned* __restrict__ epochs,
                                    int rank, int world, const T* __restrict__ weight, int rows,
                                    int hidden, float eps) {
  __shared__ float red[32];
  __shared__ unsigned s_e;
  const int per = (rows + world - 1) / world;
  const int nvec = hidden / VEC;
  const bool mine = threadIdx.x < nvec;  // one vector per thread (hidden <= 1024 * VEC)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // The grid is at most what fits on the GPU at once (every CTA resident), so
  // a CTA waiting on a peer never blocks the CTA that the peer waits for.
  for (int b = blockIdx.x; b < per; b += gridDim.x) {
    if (threadIdx.x == 0) s_e = epochs[b] + 1;
    __syncthreads();
    const unsigned e = s_e;
    if (!ar_barrier(P, 0, b, rank, world, e)) {
      if (threadIdx.x == 0) set_error(kErrTimeout);
      return;
    }
    const int row = rank * per + b;
    if (row < rows) {  // uniform over the CTA
      const int64_t off = (int64_t)row * hidden + threadIdx.x * VEC;
      float ss = 0.f;
      T hv[VEC];
      if (mine) {
        // all ranks' vectors in flight at once, then summed in rank order
        uint4 raw[kArMaxRanks];
#pragma unroll
        for (int p = 0; p < kArMaxRanks; ++p)
          if (p < world)
            raw[p] = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(P.part[p]) + off);
        T rv[VEC];
        *reinterpret_cast<uint4*>(rv) =
            *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(P.res[rank]) + off);
        float acc[VEC];
#pragma unroll
        for (int k = 0; k < VEC; ++k) acc[k] = 0.f;
#pragma unroll
        for (int p = 0; p < kArMaxRanks; ++p) {
          if (p < world) {
            const T* v = reinterpret_cast<const T*>(&raw[p]);
#pragma unroll
            for (int k = 0; k < VEC; ++k) acc[k] = __fadd_rn(acc[k], Dt<T>::to_f(v[k]));
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
      ss = warp_sum(ss);
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
        T wv[VEC], ov[VEC];
        *reinterpret_cast<uint4*>(wv) =
            __ldg(reinterpret_cast<const uint4*>(weight + threadIdx.x * VEC));
#pragma unroll
        for (int k = 0; k < VEC; ++k) {
          const float xn = Dt<T>::round(__fmul_rn(Dt<T>::to_f(hv[k]), r));
          ov[k] = Dt<T>::from_f(__fmul_rn(Dt<T>::to_f(wv[k]), xn));
        }
        const uint4 h4 = *reinterpret_cast<uint4*>(hv), o4 = *reinterpret_cast<uint4*>(ov);
#pragma unroll
        for (int p = 0; p < kArMaxRanks; ++p) {
          if (p < world) {
            *reinterpret_cast<uint4*>(reinterpret_cast<T*>(P.res[p]) + off) = h4;
            *reinterpret_cast<uint4*>(reinterpret_cast<T*>(P.out[p]) + off) = o4;
          }
        }
        __threadfence_system();  // this thread's peer stores before the CTA's release
      }
    }
    __syncthreads();
    if (!ar_barrier(P, 1, b, rank, world, e)) {
      if (threadIdx.x == 0) set_error(kErrTimeout);
      return;
    }
    if (threadIdx.x == 0) epochs[b] = e;
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

int nb_tp_allreduce_add_rmsnorm(const void* const* partials, void* const* outs,
                                void* const* residuals, unsigned* const* flags,
                                unsigned* epochs, int rank, int world, const void* weight,
                                int num_tokens, int hidden, float eps, int dtype, void* stream) {
  using namespace nbh;
  if (!valid_dtype(dtype) || dtype == NB_DTYPE_F32)
    return fail(NB_ERR_UNSUPPORTED, "fused TP all-reduce supports bf16/fp16");
  if (!partials || !outs || !residuals || !flags || !epochs || !weight)
    return fail(NB_ERR_INVALID_ARG, "null pointer argument");
  if (world < 1 || world > nb::kArMaxRanks || rank < 0 || rank >= world)
    return fail(NB_ERR_INVALID_ARG, "rank %d / world %d out of range", rank, world);
  if (num_tokens < 0 || hidden <= 0 || hidden % 8 || hidden > 1024 * 8)
    return fail(NB_ERR_UNSUPPORTED, "hidden must be a multiple of 8 up to 8192");
  const int per = (num_tokens + world - 1) / world;
  if (per > nb::kArMaxCtas)
    return fail(NB_ERR_UNSUPPORTED, "%d rows per rank exceed %d", per, nb::kArMaxCtas);
  if (num_tokens == 0) return NB_OK;
  nb::ArPeers P;
  for (int p = 0; p < world; ++p) {
    if (!partials[p] || !outs[p] || !residuals[p] || !flags[p])
      return fail(NB_ERR_INVALID_ARG, "rank %d: null buffer", p);
    P.part[p] = partials[p];
    P.out[p] = outs[p];
    P.res[p] = residuals[p];
    P.flags[p] = flags[p];
  }
  if ((uintptr_t)weight % 16) return fail(NB_ERR_INVALID_ARG, "weight must be 16-byte aligned");
  const int threads = std::max(32, ((hidden / 8 + 31) / 32) * 32);
  cudaStream_t st = (cudaStream_t)stream;
  auto launch = [&](auto kern, const auto* w) {
    // at most one resident wave: every CTA runs concurrently with its peers
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, threads, 0) != cudaSuccess ||
        occ < 1)
      return fail(NB_ERR_CUDA, "occupancy query failed");
    const int grid = std::min(per, occ * num_sms());
    kern<<<grid, threads, 0, st>>>(P, epochs, rank, world, w, num_tokens, hidden, eps);
    return check_launch("tp_allreduce_add_rmsnorm");
  };
  if (dtype == NB_DTYPE_BF16)
    return launch(nb::tp_allreduce_add_rmsnorm_kernel<__nv_bfloat16, 8>,
                  (const __nv_bfloat16*)weight);
  return launch(nb::tp_allreduce_add_rmsnorm_kernel<__half, 8>, (const __half*)weight);
}

}  // extern "C"
