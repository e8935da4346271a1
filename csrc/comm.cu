// Collectives over NVLink / NVSwitch peer memory (one process per GPU; buffers
// from symmetric memory so every rank can load/store every peer's copy).
//
//   signal barrier       every rank stores an epoch into each peer's flag slot
//                        (st.release.sys) and waits, bounded, for all peers'
//                        epochs in its own slots (ld.acquire.sys)
//   all-gather copy      dst[p*chunk + k] = peer_p.src[off + k]  (ZeRO-3 per-layer
//                        parameter gather into a local slot; plain 16-byte P2P loads)
//   reduce-scatter sum   K10 front half: out[k] = sum_p peer_p.grad[off + k] (fp32,
//                        fixed rank order so every rank's shard is deterministic)
//                        fused with the sum-of-squares partials of the result;
//                        the bf16 form reads bf16 gradients (half the NVLink
//                        bytes), sums in fp32 and accumulates into the fp32 shard
//   all-reduce sum       K12: out = sum_p peer_p.buf (one-shot, each rank reduces
//                        its 1/N slice and writes it into every peer = reduce-scatter
//                        + all-gather in one kernel) fused with unscale-free Σg^2
//                        partials and the non-finite check (inf/nan propagate)
//   norm exchange        Σg^2 partials summed locally, exchanged through peer
//                        memory, then the step finaliser (global-norm clip,
//                        overflow skip, dynamic loss scale) on the device
//
// Replaces the reference's NCCLWrapper::all_reduce / all_gather /
// reduce_scatter (include/distributed/nccl_wrapper.hpp:36-98), RingAllReduce and
// TensorFusion (include/distributed/distributed_training.hpp:152-262) and the
// ZeRO-2 step (include/distributed/zero_optimizer.hpp:56-77).
// No kernel here uses TMA or multicast; every wait is bounded.
#include "common.cuh"
#include "host_util.h"
#include "lk_api.h"

namespace lk {

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until *flag >= epoch (epochs increase monotonically).
__device__ __forceinline__ bool wait_flag(const int* flag, int epoch, int* status) {
  if (ld_acquire_sys(flag) >= epoch) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i) {
      if (ld_acquire_sys(flag) >= epoch) return true;
      __nanosleep(64);
    }
    if (globaltimer() - t0 > LK_WAIT_TIMEOUT_NS) {
      if (status) atomicCAS(status, 0, LK_ERR_TIMEOUT_PEER);
      return false;
    }
  }
}

// sig_ptrs[p] = rank p's flag array [LK_SIG_SLOTS * world]; slot s of peer q
// lives at [s * world + q].
__global__ void signal_barrier_kernel(int* const* __restrict__ sig_ptrs, int rank, int world,
                                      int slot, int epoch, int* status) {
  const int p = threadIdx.x;
  __threadfence_system();  // earlier kernels' peer stores are visible before the flag
  if (p < world) st_release_sys(sig_ptrs[p] + slot * world + rank, epoch);
  __syncthreads();
  if (p < world) wait_flag(sig_ptrs[rank] + slot * world + p, epoch, status);
  __syncthreads();
}

// The same barrier with the epoch kept on the device: the kernel advances
// *epoch_ctr itself, so a captured CUDA graph can replay it (every rank runs the
// same sequence of barriers on the slot, so the counters stay equal).
__global__ void signal_barrier_dev_kernel(int* const* __restrict__ sig_ptrs, int rank, int world, int slot,
                                          int* __restrict__ epoch_ctr, int* status) {
  __shared__ int e;
  if (threadIdx.x == 0) {
    e = *epoch_ctr + 1;
    *epoch_ctr = e;
  }
  __syncthreads();
  const int p = threadIdx.x;
  __threadfence_system();
  if (p < world) st_release_sys(sig_ptrs[p] + slot * world + rank, e);
  __syncthreads();
  if (p < world) wait_flag(sig_ptrs[rank] + slot * world + p, e, status);
  __syncthreads();
}

__global__ void allgather_copy_kernel(const uint8_t* const* __restrict__ src_ptrs, int64_t src_off,
                                      int64_t chunk_bytes, uint8_t* __restrict__ dst, int world) {
  const int64_t n16 = chunk_bytes / 16;
  const int64_t total = n16 * world;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int p = (int)(idx / n16);
    const int64_t k = idx - p * n16;
    const uint4 v = *reinterpret_cast<const uint4*>(src_ptrs[p] + src_off + k * 16);
    *reinterpret_cast<uint4*>(dst + (int64_t)p * chunk_bytes + k * 16) = v;
  }
}

template <int MAXW>
__global__ void __launch_bounds__(256) reduce_scatter_kernel(const float* const* __restrict__ src_ptrs,
                                                             int64_t src_off, int64_t n,
                                                             float* __restrict__ dst, int world,
                                                             int accumulate, float* __restrict__ partial) {
  __shared__ float red[8];
  const float* src[MAXW];
#pragma unroll
  for (int p = 0; p < MAXW; ++p) src[p] = p < world ? src_ptrs[p] + src_off : nullptr;
  float ss = 0.f;
  const int64_t n4 = n / 4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int p = 0; p < MAXW; ++p) {
      if (p >= world) break;
      const float4 v = reinterpret_cast<const float4*>(src[p])[i];
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    float4* d = reinterpret_cast<float4*>(dst) + i;
    if (accumulate) {
      const float4 o = *d;
      acc.x += o.x;
      acc.y += o.y;
      acc.z += o.z;
      acc.w += o.w;
    }
    *d = acc;
    ss += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
  }
  if (partial) {
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.f;
      for (int k = 0; k < 8; ++k) t += red[k];
      partial[blockIdx.x] = t;
    }
  }
}

// One-shot all-reduce: rank r reduces slice r (fixed peer order) and stores it
// into every peer's buffer.  Caller brackets it with signal barriers: before
// (all inputs ready) and after (all slices written).
template <int MAXW>
__global__ void __launch_bounds__(256) allreduce_kernel(float* const* __restrict__ buf_ptrs, int64_t n,
                                                        int rank, int world, float* __restrict__ partial) {
  __shared__ float red[8];
  const int64_t n4 = n / 4;
  const int64_t per = (n4 + world - 1) / world;
  const int64_t lo = rank * per, hi = min(n4, lo + per);
  float ss = 0.f;
  for (int64_t i = lo + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < hi;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int p = 0; p < MAXW; ++p) {
      if (p >= world) break;
      const float4 v = reinterpret_cast<const float4*>(buf_ptrs[p])[i];
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    ss += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
#pragma unroll
    for (int p = 0; p < MAXW; ++p) {
      if (p >= world) break;
      reinterpret_cast<float4*>(buf_ptrs[p])[i] = acc;
    }
  }
  if (partial) {
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.f;
      for (int k = 0; k < 8; ++k) t += red[k];
      partial[blockIdx.x] = t;
    }
  }
}

// Sum local partials, exchange with peers, finalise the optimizer step.
// nbuf_ptrs[p] = rank p's double[world] exchange array; flags in sig slot.
__global__ void norm_exchange_kernel(const float* __restrict__ partial, int nparts,
                                     double* const* __restrict__ nbuf_ptrs, int* const* __restrict__ sig_ptrs,
                                     int rank, int world, int slot, int epoch, float* state,
                                     float max_norm, int dynamic, float growth, float backoff,
                                     int growth_interval, float min_scale, int* status) {
  __shared__ double red[256];
  double s = 0.0;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) s += (double)partial[i];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
    __syncthreads();
  }
  const double mine = red[0];
  __syncthreads();
  if (threadIdx.x < world) {
    const int p = threadIdx.x;
    volatile double* dst = nbuf_ptrs[p] + rank;
    *dst = mine;
    __threadfence_system();
    st_release_sys(sig_ptrs[p] + slot * world + rank, epoch);
  }
  __syncthreads();
  bool ok = true;
  if (threadIdx.x < world) ok = wait_flag(sig_ptrs[rank] + slot * world + threadIdx.x, epoch, status);
  ok = __syncthreads_and(ok);
  if (threadIdx.x != 0) return;
  double tot = 0.0;
  for (int p = 0; p < world; ++p) tot += reinterpret_cast<volatile double*>(nbuf_ptrs[rank])[p];
  if (!ok) tot = NAN;  // a missing peer makes the step an overflow step (skipped)
  const float scale = state[LK_ST_LOSS_SCALE];
  const bool overflow = !isfinite(tot);
  const float norm = overflow ? INFINITY : (float)(sqrt(tot) / (double)scale);
  state[LK_ST_GRAD_NORM] = norm;
  if (overflow) {
    state[LK_ST_SKIP] = 1.f;
    state[LK_ST_NUM_SKIPPED] += 1.f;
    state[LK_ST_CONSEC_SKIPS] += 1.f;
    if (dynamic) state[LK_ST_LOSS_SCALE] = fmaxf(scale * backoff, min_scale);
    state[LK_ST_GROWTH_TRACKER] = 0.f;
    return;
  }
  const float clip = (max_norm > 0.f && norm > max_norm) ? max_norm / (norm + 1e-6f) : 1.f;
  state[LK_ST_CLIP_COEF] = clip;
  state[LK_ST_GRAD_MULT] = clip / scale;
  state[LK_ST_SKIP] = 0.f;
  state[LK_ST_CONSEC_SKIPS] = 0.f;
  state[LK_ST_STEP] += 1.f;
  if (dynamic) {
    const float t = state[LK_ST_GROWTH_TRACKER] + 1.f;
    if (t >= (float)growth_interval) {
      state[LK_ST_LOSS_SCALE] = scale * growth;
      state[LK_ST_GROWTH_TRACKER] = 0.f;
    } else {
      state[LK_ST_GROWTH_TRACKER] = t;
    }
  }
}

// ------------------------------------------------------------------ NVLS
// The same two reductions through the NVSwitch: a multicast address maps
// every rank's copy of the buffer; multimem.ld_reduce returns the sum over all
// ranks (reduced inside the switch) and multimem.st writes one value into
// every rank's copy.  Each rank moves 1/world of the data once in each
// direction instead of pulling every peer's copy.
__device__ __forceinline__ float4 mm_ld_reduce_add(const float* mc) {
  float4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}

__device__ __forceinline__ void mm_st(float* mc, float4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}

__device__ __forceinline__ void block_partial(float ss, float* partial) {
  __shared__ float red[8];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int k = 0; k < 8; ++k) t += red[k];
    partial[blockIdx.x] = t;
  }
}

__global__ void __launch_bounds__(256) allreduce_nvls_kernel(float* __restrict__ mc, int64_t n, int rank,
                                                             int world, float* __restrict__ partial) {
  const int64_t n4 = n / 4;
  const int64_t per = (n4 + world - 1) / world;
  const int64_t lo = rank * per, hi = min(n4, lo + per);
  float ss = 0.f;
  for (int64_t i = lo + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < hi;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = mm_ld_reduce_add(mc + 4 * i);
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    mm_st(mc + 4 * i, v);
  }
  if (partial) block_partial(ss, partial);
}

__global__ void __launch_bounds__(256) reduce_scatter_nvls_kernel(const float* __restrict__ mc, int64_t n,
                                                                  float* __restrict__ dst, int accumulate,
                                                                  float* __restrict__ partial) {
  float ss = 0.f;
  const int64_t n4 = n / 4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 acc = mm_ld_reduce_add(mc + 4 * i);
    float4* d = reinterpret_cast<float4*>(dst) + i;
    if (accumulate) {
      const float4 o = *d;
      acc.x += o.x;
      acc.y += o.y;
      acc.z += o.z;
      acc.w += o.w;
    }
    *d = acc;
    ss += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
  }
  if (partial) block_partial(ss, partial);
}

// ZeRO gradient reduce-scatter with bf16 on the wire (K10): every rank's
// gradients of a layer group sit in a bf16 slot of symmetric memory; the owner
// of a chunk loads the peers' bf16 values, sums them in fp32 in a fixed rank
// order, adds the result into its fp32 gradient shard (or stores it on the
// first micro-batch of an accumulation window) and emits the sum-of-squares
// partials of the shard when asked (last micro-batch).  Half the bytes of the
// fp32 exchange cross NVLink.
template <int MAXW>
__global__ void __launch_bounds__(256) reduce_scatter_bf16_kernel(
    const __nv_bfloat16* const* __restrict__ src_ptrs, int64_t src_off, int64_t n, float* __restrict__ dst,
    int world, int accumulate, float* __restrict__ partial) {
  const __nv_bfloat16* src[MAXW];
#pragma unroll
  for (int p = 0; p < MAXW; ++p) src[p] = p < world ? src_ptrs[p] + src_off : nullptr;
  float ss = 0.f;
  const int64_t n8 = n / 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8;
       i += (int64_t)gridDim.x * blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int p = 0; p < MAXW; ++p) {
      if (p >= world) break;
      const uint4 v = reinterpret_cast<const uint4*>(src[p])[i];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack_bf16x2(w[e]);
        acc[2 * e] += f.x;
        acc[2 * e + 1] += f.y;
      }
    }
    float4* d = reinterpret_cast<float4*>(dst) + 2 * i;
    float4 o0 = make_float4(acc[0], acc[1], acc[2], acc[3]);
    float4 o1 = make_float4(acc[4], acc[5], acc[6], acc[7]);
    if (accumulate) {
      const float4 a = d[0], b = d[1];
      o0.x += a.x; o0.y += a.y; o0.z += a.z; o0.w += a.w;
      o1.x += b.x; o1.y += b.y; o1.z += b.z; o1.w += b.w;
    }
    d[0] = o0;
    d[1] = o1;
    ss += o0.x * o0.x + o0.y * o0.y + o0.z * o0.z + o0.w * o0.w + o1.x * o1.x + o1.y * o1.y + o1.z * o1.z +
          o1.w * o1.w;
  }
  if (partial) {
    __shared__ float red[8];
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.f;
      for (int k = 0; k < 8; ++k) t += red[k];
      partial[blockIdx.x] = t;
    }
  }
}

// NVLS form: the switch adds the ranks' bf16 values with fp32 accumulation
// (one rounding of the sum to bf16), then the owner accumulates in fp32.
__device__ __forceinline__ uint4 mm_ld_reduce_bf16x8(const __nv_bfloat16* mc) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}

__global__ void __launch_bounds__(256) reduce_scatter_bf16_nvls_kernel(const __nv_bfloat16* __restrict__ mc,
                                                                       int64_t n, float* __restrict__ dst,
                                                                       int accumulate, float* __restrict__ partial) {
  float ss = 0.f;
  const int64_t n8 = n / 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 v = mm_ld_reduce_bf16x8(mc + 8 * i);
    const float2 a = unpack_bf16x2(v.x), b = unpack_bf16x2(v.y), c = unpack_bf16x2(v.z), e = unpack_bf16x2(v.w);
    float4 o0 = make_float4(a.x, a.y, b.x, b.y);
    float4 o1 = make_float4(c.x, c.y, e.x, e.y);
    float4* d = reinterpret_cast<float4*>(dst) + 2 * i;
    if (accumulate) {
      const float4 p0 = d[0], p1 = d[1];
      o0.x += p0.x; o0.y += p0.y; o0.z += p0.z; o0.w += p0.w;
      o1.x += p1.x; o1.y += p1.y; o1.z += p1.z; o1.w += p1.w;
    }
    d[0] = o0;
    d[1] = o1;
    ss += o0.x * o0.x + o0.y * o0.y + o0.z * o0.z + o0.w * o0.w + o1.x * o1.x + o1.y * o1.y + o1.z * o1.z +
          o1.w * o1.w;
  }
  if (partial) block_partial(ss, partial);
}

static int copy_grid(int64_t work) {
  int64_t g = (work + 255) / 256;
  const int64_t cap = (int64_t)num_sms() * 4;
  return (int)(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace lk

using namespace lk;

extern "C" int lk_signal_barrier(int* const* sig_ptrs, int rank, int world, int slot, int epoch,
                                 int* status, cudaStream_t s) {
  LK_REQUIRE(world >= 1 && world <= 32 && slot >= 0 && slot < LK_SIG_SLOTS, "signal_barrier: bad args");
  signal_barrier_kernel<<<1, 32, 0, s>>>(sig_ptrs, rank, world, slot, epoch, status);
  return check_launch("signal_barrier");
}

extern "C" int lk_signal_barrier_dev(int* const* sig_ptrs, int rank, int world, int slot, int* epoch_ctr,
                                     int* status, cudaStream_t s) {
  LK_REQUIRE(world >= 1 && world <= 32 && slot >= 0 && slot < LK_SIG_SLOTS && epoch_ctr,
             "signal_barrier_dev: bad args");
  signal_barrier_dev_kernel<<<1, 32, 0, s>>>(sig_ptrs, rank, world, slot, epoch_ctr, status);
  return check_launch("signal_barrier_dev");
}

extern "C" int lk_allgather_copy(const void* const* src_ptrs, int64_t src_off_bytes,
                                 int64_t chunk_bytes, void* dst, int world, cudaStream_t s) {
  LK_REQUIRE(src_off_bytes % 16 == 0 && chunk_bytes % 16 == 0, "allgather_copy: 16-byte alignment");
  if (chunk_bytes == 0) return 0;
  allgather_copy_kernel<<<copy_grid(chunk_bytes / 16 * world), 256, 0, s>>>(
      (const uint8_t* const*)src_ptrs, src_off_bytes, chunk_bytes, (uint8_t*)dst, world);
  return check_launch("allgather_copy");
}

extern "C" int lk_reduce_scatter_sum(const float* const* src_ptrs, int64_t src_off, int64_t n,
                                     float* dst, int world, int accumulate, float* partial,
                                     int nparts, cudaStream_t s) {
  LK_REQUIRE(world >= 1 && world <= 8, "reduce_scatter: world must be 1..8");
  LK_REQUIRE(n % 4 == 0 && src_off % 4 == 0, "reduce_scatter: sizes must be multiples of 4");
  if (n == 0) return 0;
  int grid = copy_grid(n / 4);
  if (partial) grid = nparts < grid ? nparts : grid;
  reduce_scatter_kernel<8><<<grid, 256, 0, s>>>(src_ptrs, src_off, n, dst, world, accumulate, partial);
  if (partial && nparts > grid) cudaMemsetAsync(partial + grid, 0, sizeof(float) * (nparts - grid), s);
  return check_launch("reduce_scatter_sum");
}

extern "C" int lk_allreduce_sum(float* const* buf_ptrs, int64_t n, int rank, int world,
                                float* partial, int nparts, cudaStream_t s) {
  LK_REQUIRE(world >= 1 && world <= 8, "allreduce: world must be 1..8");
  LK_REQUIRE(n % 4 == 0, "allreduce: n must be a multiple of 4");
  int grid = copy_grid((n / 4 + world - 1) / world);
  if (partial) grid = nparts < grid ? nparts : grid;
  allreduce_kernel<8><<<grid, 256, 0, s>>>(buf_ptrs, n, rank, world, partial);
  if (partial && nparts > grid) cudaMemsetAsync(partial + grid, 0, sizeof(float) * (nparts - grid), s);
  return check_launch("allreduce_sum");
}

extern "C" int lk_norm_exchange(const float* partial, int nparts, double* const* nbuf_ptrs,
                                int* const* sig_ptrs, int rank, int world, int slot, int epoch,
                                float* state, float max_norm, int dynamic, float growth,
                                float backoff, int growth_interval, float min_scale, int* status,
                                cudaStream_t s) {
  LK_REQUIRE(world >= 1 && world <= 32, "norm_exchange: bad world");
  norm_exchange_kernel<<<1, 256, 0, s>>>(partial, nparts, nbuf_ptrs, sig_ptrs, rank, world, slot,
                                         epoch, state, max_norm, dynamic, growth, backoff,
                                         growth_interval, min_scale, status);
  return check_launch("norm_exchange");
}

extern "C" int lk_allreduce_sum_nvls(float* mc, int64_t n, int rank, int world, float* partial, int nparts,
                                     cudaStream_t s) {
  LK_REQUIRE(mc && n % 4 == 0 && ((uintptr_t)mc & 15) == 0, "allreduce_nvls: aligned multicast buffer, n % 4");
  int grid = copy_grid((n / 4 + world - 1) / world);
  if (partial) grid = nparts < grid ? nparts : grid;
  allreduce_nvls_kernel<<<grid, 256, 0, s>>>(mc, n, rank, world, partial);
  if (partial && nparts > grid) cudaMemsetAsync(partial + grid, 0, sizeof(float) * (nparts - grid), s);
  return check_launch("allreduce_nvls");
}

extern "C" int lk_reduce_scatter_sum_nvls(const float* mc, int64_t n, float* dst, int accumulate, float* partial,
                                          int nparts, cudaStream_t s) {
  LK_REQUIRE(mc && n % 4 == 0 && ((uintptr_t)mc & 15) == 0, "reduce_scatter_nvls: aligned multicast buffer");
  int grid = copy_grid(n / 4);
  if (partial) grid = nparts < grid ? nparts : grid;
  reduce_scatter_nvls_kernel<<<grid, 256, 0, s>>>(mc, n, dst, accumulate, partial);
  if (partial && nparts > grid) cudaMemsetAsync(partial + grid, 0, sizeof(float) * (nparts - grid), s);
  return check_launch("reduce_scatter_nvls");
}

extern "C" int lk_reduce_scatter_bf16(const void* const* src_ptrs, int64_t src_off, int64_t n, float* dst,
                                      int world, int accumulate, float* partial, int nparts, cudaStream_t s) {
  LK_REQUIRE(world >= 1 && world <= 8, "reduce_scatter_bf16: world must be 1..8");
  LK_REQUIRE(n % 8 == 0 && src_off % 8 == 0 && ((uintptr_t)dst & 15) == 0,
             "reduce_scatter_bf16: n and offset must be multiples of 8, dst 16-byte aligned");
  if (n == 0) return 0;
  int grid = copy_grid(n / 8);
  if (partial) grid = nparts < grid ? nparts : grid;
  reduce_scatter_bf16_kernel<8><<<grid, 256, 0, s>>>((const __nv_bfloat16* const*)src_ptrs, src_off, n, dst,
                                                     world, accumulate, partial);
  if (partial && nparts > grid) cudaMemsetAsync(partial + grid, 0, sizeof(float) * (nparts - grid), s);
  return check_launch("reduce_scatter_bf16");
}

extern "C" int lk_reduce_scatter_bf16_nvls(const void* mc, int64_t n, float* dst, int accumulate, float* partial,
                                           int nparts, cudaStream_t s) {
  LK_REQUIRE(mc && n % 8 == 0 && ((uintptr_t)mc & 15) == 0 && ((uintptr_t)dst & 15) == 0,
             "reduce_scatter_bf16_nvls: 16-byte aligned buffers, n % 8");
  if (n == 0) return 0;
  int grid = copy_grid(n / 8);
  if (partial) grid = nparts < grid ? nparts : grid;
  reduce_scatter_bf16_nvls_kernel<<<grid, 256, 0, s>>>((const __nv_bfloat16*)mc, n, dst, accumulate, partial);
  if (partial && nparts > grid) cudaMemsetAsync(partial + grid, 0, sizeof(float) * (nparts - grid), s);
  return check_launch("reduce_scatter_bf16_nvls");
}
