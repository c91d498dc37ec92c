// Split-context merge over NVLink peer memory (no collective library).
//
// In split-context decode every GPU computes, for the whole batch, a
// log-sum-exp partial (O [rows, D] fp32 normalised, lse [rows] fp32) over the
// context splits it holds, and every GPU needs the merge of all of them.
// Instead of an all-gather followed by a merge, one kernel per GPU and step
// publishes this GPU's partial in an exchange buffer the other GPUs have
// mapped (CUDA IPC), then reads every GPU's partial from its owner's memory
// over NVLink and writes the merged fp16 output.  The data crosses NVLink
// once, inside the kernel that consumes it; a step is the decode plus this
// one kernel.
//
// Exchange buffer of one GPU (cudaMalloc'ed, zeroed, mapped by the peers):
//   header (256 B): [0]   flag  = the last step whose partial is published
//                                 (system-scope release by the owner)
//                   [64]  epoch = the owner's step counter
//                   [128] count = CTA arrivals of the running merge
//   then two slots, each O [rows, D] fp32 and lse [rows] fp32.
// Step e of the merge on one GPU (a cooperative launch: all CTAs resident):
// every CTA copies its share of the GPU's partial into slot e & 1; the last
// CTA to finish raises the flag to e; every CTA waits until every GPU's flag
// reaches e (its own included) and merges its rows from slot e & 1 of every
// buffer.  Slot e & 1 is written again at step e + 2, after this GPU's merge
// of e + 1 saw every peer's flag reach e + 1, which each peer raised only
// after its merge of e had read the slot: no peer reads a slot while it is
// rewritten, and none waits for the others to finish reading.  Every GPU runs
// the merge once per step, in the same order.  Waits are bounded: a GPU that
// does not arrive within the limit makes the merge set
// IRIS_ERR_PIPELINE_TIMEOUT (the exchange must then be rebuilt).  No
// multicast, no library kernel on peer memory.
#include <cstring>

#include "common.cuh"

namespace {

constexpr int kMaxRanks = 8;
constexpr int kXchgThreads = 256;

struct Header {
  unsigned long long flag;
  unsigned long long pad0[7];
  unsigned long long epoch;
  unsigned long long pad1[7];
  unsigned int count;
};
static_assert(sizeof(Header) <= IRIS_XCHG_HEADER_BYTES, "exchange header");

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Spin until *p >= want, at most limit_ns after t0; false when it gave up.
__device__ __forceinline__ bool wait_at_least(const unsigned long long* p, unsigned long long want, uint64_t t0,
                                              uint64_t limit_ns) {
  while (ld_acquire_sys(p) < want) {
    if (iris::globaltimer_ns() - t0 > limit_ns) return false;
    __nanosleep(64);
  }
  return true;
}

struct Peers {
  uint8_t* buf[kMaxRanks];
};

// Bytes of one slot (O then lse), rounded to 256 so that slot 1 is aligned too.
__host__ __device__ inline size_t slot_bytes(int64_t rows, int32_t head_dim) {
  return (static_cast<size_t>(rows) * (head_dim + 1) * 4 + 255) & ~static_cast<size_t>(255);
}

// One warp per row, 4 dims per lane and step; NR (the number of GPUs, a
// compile-time constant) lets every GPU's loads of a row issue together, and
// the first 128 dims' O values are loaded with the lse values, so a row of
// head_dim <= 128 costs one NVLink round trip.  A part with lse = -inf holds
// none of the row's tokens and is skipped (its O may hold anything).
template <int NR>
__global__ void __launch_bounds__(kXchgThreads) xchg_merge_kernel(Peers peers, int32_t me, int64_t rows,
                                                                  int32_t head_dim, const float* __restrict__ lo,
                                                                  const float* __restrict__ llse,
                                                                  __half* __restrict__ out, int32_t* err,
                                                                  uint64_t limit_ns) {
  __shared__ int ok;
  Header* mine = reinterpret_cast<Header*>(peers.buf[me]);
  const unsigned long long e = *reinterpret_cast<volatile unsigned long long*>(&mine->epoch) + 1;
  const int64_t n_o = rows * head_dim;
  const size_t slot = IRIS_XCHG_HEADER_BYTES + (e & 1) * slot_bytes(rows, head_dim);
  const uint64_t t0 = iris::globaltimer_ns();
  // publish this GPU's partial in slot e & 1
  {
    float* dst = reinterpret_cast<float*>(peers.buf[me] + slot);
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n_o / 4; i += stride)
      reinterpret_cast<float4*>(dst)[i] = reinterpret_cast<const float4*>(lo)[i];
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < rows; i += stride)
      dst[n_o + i] = llse[i];
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int done = atomicAdd(&mine->count, 1u);
    if (done == gridDim.x - 1) {  // every CTA's copy is done (each fenced before arriving)
      __threadfence();
      mine->count = 0;
      mine->epoch = e;              // every CTA has read the epoch: it arrived above
      st_release_sys(&mine->flag, e);  // the slot is visible to whoever acquires e
    }
  }
  if (threadIdx.x < 32) {  // lane k waits for GPU k's flag (its own included: every CTA's copy)
    int good = 1;
    if (threadIdx.x < NR)
      good = wait_at_least(&reinterpret_cast<const Header*>(peers.buf[threadIdx.x])->flag, e, t0, limit_ns);
    const unsigned all = __ballot_sync(0xffffffffu, good);
    if (threadIdx.x == 0) ok = all == 0xffffffffu;
  }
  __syncthreads();
  if (!ok) {
    if (threadIdx.x == 0) iris::set_error(err, IRIS_ERR_PIPELINE_TIMEOUT);
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const float kNegInf = -__int_as_float(0x7f800000);
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * warps + warp; row < rows;
       row += static_cast<int64_t>(gridDim.x) * warps) {
    float lse[NR];
    float4 v[NR];
#pragma unroll
    for (int k = 0; k < NR; ++k) {
      const float* part = reinterpret_cast<const float*>(peers.buf[k] + slot);
      lse[k] = __ldcv(part + n_o + row);
      if (4 * lane < head_dim) v[k] = __ldcv(reinterpret_cast<const float4*>(part + row * head_dim + 4 * lane));
    }
    float mx = kNegInf;
#pragma unroll
    for (int k = 0; k < NR; ++k) mx = fmaxf(mx, lse[k]);
    for (int d = 4 * lane; d < head_dim; d += 128) {
      if (d != 4 * lane) {
#pragma unroll
        for (int k = 0; k < NR; ++k)
          v[k] = __ldcv(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(peers.buf[k] + slot) +
                                                        row * head_dim + d));
      }
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      float ws = 0.f;
#pragma unroll
      for (int k = 0; k < NR; ++k) {
        const bool has = lse[k] != kNegInf;
        const float w = has ? iris::ex2(lse[k] - mx) : 0.f;
        const float4 x = has ? v[k] : make_float4(0.f, 0.f, 0.f, 0.f);
        acc.x = fmaf(w, x.x, acc.x);
        acc.y = fmaf(w, x.y, acc.y);
        acc.z = fmaf(w, x.z, acc.z);
        acc.w = fmaf(w, x.w, acc.w);
        ws += w;
      }
      const float inv = 1.0f / ws;
      uint2 u;
      u.x = iris::h2_as_u32(__floats2half2_rn(acc.x * inv, acc.y * inv));
      u.y = iris::h2_as_u32(__floats2half2_rn(acc.z * inv, acc.w * inv));
      *reinterpret_cast<uint2*>(out + row * head_dim + d) = u;
    }
  }
}

}  // namespace

extern "C" size_t iris_b200_xchg_buffer_bytes(int64_t rows, int32_t head_dim) {
  if (rows <= 0 || head_dim <= 0 || head_dim % 4 != 0) return 0;
  return IRIS_XCHG_HEADER_BYTES + 2 * slot_bytes(rows, head_dim);
}

extern "C" int iris_b200_xchg_alloc(size_t bytes, void** buf) {
  if (buf == nullptr || bytes < static_cast<size_t>(IRIS_XCHG_HEADER_BYTES)) return IRIS_EINVAL;
  iris::clear_stale_cuda_error();
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    iris::record_cuda_error(e, "exchange buffer allocation");
    if (p != nullptr) cudaFree(p);
    return IRIS_ECUDA;
  }
  *buf = p;
  return IRIS_OK;
}

extern "C" int iris_b200_xchg_free(void* buf) {
  if (buf == nullptr) return IRIS_OK;
  const cudaError_t e = cudaFree(buf);
  if (e != cudaSuccess) {
    iris::record_cuda_error(e, "cudaFree(exchange buffer)");
    return IRIS_ECUDA;
  }
  return IRIS_OK;
}

extern "C" int iris_b200_ipc_export(const void* buf, void* handle) {
  if (buf == nullptr || handle == nullptr) return IRIS_EINVAL;
  iris::clear_stale_cuda_error();
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(buf));
  if (e != cudaSuccess) {
    iris::record_cuda_error(e, "cudaIpcGetMemHandle");
    return IRIS_ECUDA;
  }
  static_assert(sizeof(h) == IRIS_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  return IRIS_OK;
}

extern "C" int iris_b200_ipc_open(const void* handle, void** peer_buf) {
  if (handle == nullptr || peer_buf == nullptr) return IRIS_EINVAL;
  iris::clear_stale_cuda_error();
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    iris::record_cuda_error(e, "cudaIpcOpenMemHandle");
    return IRIS_ECUDA;
  }
  *peer_buf = p;
  return IRIS_OK;
}

extern "C" int iris_b200_ipc_close(void* peer_buf) {
  if (peer_buf == nullptr) return IRIS_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(peer_buf);
  if (e != cudaSuccess) {
    iris::record_cuda_error(e, "cudaIpcCloseMemHandle");
    return IRIS_ECUDA;
  }
  return IRIS_OK;
}

extern "C" int iris_b200_xchg_merge(void* const* bufs, int32_t num_ranks, int32_t my_rank, int64_t rows,
                                    int32_t head_dim, const float* local_o, const float* local_lse, void* output,
                                    int32_t* error_word, int64_t limit_ns, void* stream) {
  if (bufs == nullptr || local_o == nullptr || local_lse == nullptr || output == nullptr || num_ranks <= 0 ||
      num_ranks > kMaxRanks || my_rank < 0 || my_rank >= num_ranks || rows <= 0 || head_dim <= 0 ||
      head_dim % 4 != 0 || head_dim > 512 || limit_ns <= 0)
    return IRIS_EINVAL;
  Peers peers = {};
  for (int k = 0; k < num_ranks; ++k) {
    if (bufs[k] == nullptr || reinterpret_cast<uintptr_t>(bufs[k]) % 256 != 0) return IRIS_EALIGN;
    peers.buf[k] = static_cast<uint8_t*>(bufs[k]);
  }
  if (reinterpret_cast<uintptr_t>(output) % 8 != 0 || reinterpret_cast<uintptr_t>(local_o) % 16 != 0 ||
      reinterpret_cast<uintptr_t>(local_lse) % 4 != 0)
    return IRIS_EALIGN;
  iris::clear_stale_cuda_error();
  int device = 0, sms = 0;
  if (cudaGetDevice(&device) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || sms <= 0) {
    iris::record_cuda_error(cudaGetLastError(), "xchg_merge device query");
    return IRIS_ECUDA;
  }
  // at most one CTA per SM: a cooperative launch, every CTA resident (each waits for the others' copies)
  const int64_t need = (rows + kXchgThreads / 32 - 1) / (kXchgThreads / 32);
  const int grid = static_cast<int>(need < sms ? need : sms);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kXchgThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  __half* out = static_cast<__half*>(output);
  const uint64_t lim = static_cast<uint64_t>(limit_ns);
  cudaError_t e = cudaSuccess;
  switch (num_ranks) {  // one instance per GPU count
#define IRIS_XCHG_CASE(N)                                                                                  \
  case N:                                                                                                  \
    e = cudaLaunchKernelEx(&cfg, xchg_merge_kernel<N>, peers, my_rank, rows, head_dim, local_o, local_lse, out, \
                           error_word, lim);                                                               \
    break;
    IRIS_XCHG_CASE(1)
    IRIS_XCHG_CASE(2)
    IRIS_XCHG_CASE(3)
    IRIS_XCHG_CASE(4)
    IRIS_XCHG_CASE(5)
    IRIS_XCHG_CASE(6)
    IRIS_XCHG_CASE(7)
    IRIS_XCHG_CASE(8)
#undef IRIS_XCHG_CASE
    default:
      return IRIS_EUNSUPPORTED;
  }
  if (e != cudaSuccess) {
    iris::record_cuda_error(e, "xchg_merge_kernel launch");
    return IRIS_ECUDA;
  }
  return IRIS_OK;
}
