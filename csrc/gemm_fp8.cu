// K2: block-scaled fp8 GEMM on the 5th-generation tensor cores.
//
//   D[m, n] = sum_kb  sa[kb, m] * sb[n / 128, kb] * sum_{k in block kb} A8[m, k] * B8[n, k]
//
// A (activations or output gradients): fp8 e4m3 or e5m2, one fp32 scale per row
// and 128-wide K block (1 x 128).  B (weights): fp8 e4m3, one fp32 scale per
// 128 x 128 block.  Each 128-element K block is contracted by four
// tcgen05.mma.kind::f8f6f4 (K = 32 each) into a fresh fp32 TMEM partial; the
// epilogue warps read the partial back (tcgen05.ld), scale it by
// sa[m] * sb and add it to the row's fp32 accumulator in registers, so the
// block scales are applied exactly (DeepSeek-V3 style promotion, with TMEM
// instead of a register accumulator).  Four TMEM partials rotate so the MMAs
// run up to four K blocks ahead of the promotion.
//
// Tile 128 x 128 (one CTA per SM, persistent), K step 128 fp8 = one 128-byte
// swizzle row, 6-stage TMA ring.  Warp 0: TMA producer; warp 1: MMA issuer;
// warps 2-5: promotion + epilogue (thread = output row).  Every wait is bounded.
//
// Reference: the reference's FP8 path is a scalar per-tensor cast around an fp32
// matmul (include/nn/mixed_precision.hpp:20-75); this is the tensor-core form.
#include "common.cuh"
#include "host_util.h"
#include "lk_api.h"

namespace lk {
namespace {

constexpr int F8_BM = 128, F8_BN = 128, F8_BK = 128;  // BK in elements (= bytes)
constexpr int F8_STAGES = 6;
constexpr int F8_STAGE = (F8_BM + F8_BN) * F8_BK;     // 32 KB
constexpr int F8_EW = 4;                     // promotion warps (4: one per TMEM lane quarter)
constexpr int F8_THREADS = 64 + 32 * F8_EW;  // + producer and MMA-issuer warps
constexpr int F8_EPI = 32 * F8_EW;           // promotion threads
constexpr int F8_NPB = 4;                    // TMEM partials in flight (4 x 128 columns)
constexpr int F8_SC_DIST = 6, F8_SC_RING = 8;  // scale prefetch distance / ring depth (K blocks)
constexpr int F8_SMEM = F8_STAGES * F8_STAGE + 256 + F8_SC_RING * F8_EPI * 8 + 1024;

// 4-byte asynchronous copy global -> shared (zero-filled when src_bytes == 0).
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

struct F8Args {
  int M, N, K;
  const float* sa;  // [K/128, M]
  const float* sb;  // [ceil(N/128), K/128]
  void* D;
  int64_t ldd;
  const __nv_bfloat16* R;  // optional residual [M, N]
  int64_t ldr;
  int* status;
  int tiles_m, tiles_n;
  // fused all-gather of A (fp8 rows + their 1x128 scales) on first use
  const uint8_t* const* ag_rows;  // per rank: ag_r rows x K fp8 (pitch K)
  const float* const* ag_scales;  // per rank: [K/128, ag_r] scales
  uint8_t* a_dst;                 // local A [M, K] (pitch K)
  float* sa_dst;                  // local sa [K/128, M] (= sa)
  int ag_r, ag_rank, ag_world;
  int* ag_count;                  // [M/128] pieces copied per 128-row chunk
  // remote-store epilogue (reduce-scatter): row m -> rptrs[m / rs_rows] at row rs_rank*rs_rows + m % rs_rows
  void* const* rptrs;
  int rs_rows, rs_rank;
};

__device__ __forceinline__ void f8_fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ int f8_ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// bounded wait for a 128-row chunk of gathered rows (8 pieces of 16 rows)
__device__ __forceinline__ bool f8_wait_chunk(const F8Args& a, int tm, volatile int* abort_flag) {
  const int* cnt = a.ag_count + tm;
  const uint64_t t0 = globaltimer();
  while (f8_ld_acquire(cnt) < 8) {
    if (*abort_flag) return false;
    if (globaltimer() - t0 > LK_WAIT_TIMEOUT_NS) {
      atomicCAS(a.status, 0, LK_ERR_TIMEOUT_PEER);
      *abort_flag = 1;
      return false;
    }
    __nanosleep(100);
  }
  f8_fence_proxy_async_global();
  return true;
}

// copy warps: 16-row pieces (own rows first, then rank+1, ...) of fp8 rows and their scales
__device__ __forceinline__ void f8_ag_copy(const F8Args& a, int cw, int ncw, int lane) {
  const int R = a.ag_r, W = a.ag_world, me = a.ag_rank, K = a.K, KB = a.K / 128;
  const int per_rank = R / 16;
  const int upr = K / 16;  // 16-byte units per fp8 row
  for (int s = cw; s < per_rank * W; s += ncw) {
    const int p = (me + s / per_rank) % W;
    const int r0 = (s % per_rank) * 16;
#pragma unroll 1
    for (int r = 0; r < 16; ++r) {
      const uint4* sr = reinterpret_cast<const uint4*>(a.ag_rows[p] + (int64_t)(r0 + r) * K);
      uint4* dr = reinterpret_cast<uint4*>(a.a_dst + (int64_t)(p * R + r0 + r) * K);
#pragma unroll 1
      for (int c0 = lane; c0 < upr; c0 += 32 * 8) {
        uint4 v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (c0 + 32 * k < upr) v[k] = sr[c0 + 32 * k];
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (c0 + 32 * k < upr) dr[c0 + 32 * k] = v[k];
      }
    }
    // scales of those 16 rows: KB rows of 16 floats
    for (int u = lane; u < KB * 4; u += 32) {
      const int kb = u >> 2, q4 = u & 3;
      const float4 v = *reinterpret_cast<const float4*>(a.ag_scales[p] + (int64_t)kb * R + r0 + q4 * 4);
      *reinterpret_cast<float4*>(a.sa_dst + (int64_t)kb * a.M + p * R + r0 + q4 * 4) = v;
    }
    f8_fence_proxy_async_global();
    __threadfence();
    __syncwarp();
    if (lane == 0) atomicAdd(a.ag_count + (p * R + r0) / 128, 1);
  }
}

__device__ __forceinline__ void f8_tile(int t, int tiles_m, int tiles_n, int& tm, int& tn) {
  constexpr int G = 16;
  const int group = t / (G * tiles_n);
  const int first_m = group * G;
  const int gsz = min(tiles_m - first_m, G);
  const int r = t - group * G * tiles_n;
  tm = first_m + r % gsz;
  tn = r / gsz;
}

template <int AFMT, bool AG = false, bool REMOTE = false>
__global__ void __launch_bounds__(F8_THREADS + (AG ? 64 : 0), 1)
    gemm_fp8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const F8Args args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + F8_STAGES * F8_STAGE);
  const uint32_t full0 = smem_u32(bars);
  const uint32_t empty0 = full0 + 8 * F8_STAGES;
  const uint32_t pfull0 = empty0 + 8 * F8_STAGES;  // [NPB] a TMEM partial is ready
  const uint32_t pempty0 = pfull0 + 8 * F8_NPB;    // [NPB] the epilogue has read it
  const uint32_t drain_bar = pempty0 + 8 * F8_NPB;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * F8_STAGES + 2 * F8_NPB + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < F8_STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < F8_NPB; ++b) {
      mbar_init(pfull0 + 8 * b, 1);
      mbar_init(pempty0 + 8 * b, F8_EW);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), F8_NPB * F8_BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int T = args.tiles_m * args.tiles_n;
  const int nk = args.K / F8_BK;

  if (warp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0, pending = 0, parbits = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < T && ok; t += gridDim.x) {
        int tm, tn;
        f8_tile(t, args.tiles_m, args.tiles_n, tm, tn);
        if constexpr (AG) {
          tm = (tm + args.ag_rank * (args.ag_r / F8_BM)) % args.tiles_m;  // own rows first
          if (!f8_wait_chunk(args, tm, abort_flag)) {
            ok = false;
            break;
          }
        }
        for (int kb = 0; kb < nk; ++kb) {
          if (!bounded_wait(empty0 + 8 * s, ph ^ 1, args.status, LK_ERR_TIMEOUT_EMPTY, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t fb = full0 + 8 * s;
          const uint32_t sa = sbase + s * F8_STAGE;
          mbar_expect_tx(fb, F8_STAGE);
          tma_load_2d(sa, &tmA, fb, kb * F8_BK, tm * F8_BM);
          tma_load_2d(sa + F8_BM * F8_BK, &tmB, fb, kb * F8_BK, tn * F8_BN);
          pending |= 1u << s;
          parbits = (parbits & ~(1u << s)) | (ph << s);
          if (++s == F8_STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      if (!ok)
        for (int i = 0; i < F8_STAGES; ++i)
          if (pending & (1u << i))
            bounded_wait(full0 + 8 * i, (parbits >> i) & 1, args.status, LK_ERR_TIMEOUT_DRAIN, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f8(F8_BM, F8_BN, AFMT, 0);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      uint32_t g = 0;  // K blocks issued by this CTA (selects the TMEM partial)
      for (int t = blockIdx.x; t < T && ok; t += gridDim.x) {
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const uint32_t pb = g % F8_NPB, use = g / F8_NPB;
          if (!bounded_wait(pempty0 + 8 * pb, (use & 1) ^ 1, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag) ||
              !bounded_wait(full0 + 8 * s, ph, args.status, LK_ERR_TIMEOUT_FULL, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = sbase + s * F8_STAGE;
          const uint32_t sb = sa + F8_BM * F8_BK;
#pragma unroll
          for (int kk = 0; kk < F8_BK / 32; ++kk)
            tc_mma_f8(tmem + pb * F8_BN, make_desc_sw128(sa + kk * 32, 16, 1024),
                      make_desc_sw128(sb + kk * 32, 16, 1024), idesc, kk != 0 ? 1u : 0u);
          tc_commit(empty0 + 8 * s);
          tc_commit(pfull0 + 8 * pb);
          if (++s == F8_STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      tc_commit(drain_bar);
      bounded_wait(drain_bar, 0, args.status, LK_ERR_TIMEOUT_DRAIN, nullptr);
    }
  } else if (AG && warp >= 2 + F8_EW) {
    // ---------------------------------------------------------- copy warps
    f8_ag_copy(args, (warp - 2 - F8_EW) * gridDim.x + blockIdx.x, 2 * gridDim.x, lane);
  } else {
    // ------------------------------------------- promotion + epilogue (row per thread)
    const int q = warp & 3;                 // TMEM lane quarter this warp may read
    const int half = (warp - 2) >> 2;       // which slice of the tile's columns (8 warps)
    const int et = (warp - 2) * 32 + lane;  // promotion thread id (scale ring slot)
    const int row_in_tile = q * 32 + lane;
    constexpr int HN = F8_BN * 4 / F8_EW;   // columns per thread
    const int nkb_b = nk;  // sb row length
    // per-thread ring of (sa, sb) scale pairs, filled F8_SC_DIST K blocks ahead with cp.async
    const uint32_t sring = sbase + F8_STAGES * F8_STAGE + 256;
    uint32_t g = 0;
    for (int t = blockIdx.x; t < T; t += gridDim.x) {
      int tm, tn;
      f8_tile(t, args.tiles_m, args.tiles_n, tm, tn);
      if constexpr (AG) {
        tm = (tm + args.ag_rank * (args.ag_r / F8_BM)) % args.tiles_m;
        // the tile's row scales come with the gathered rows: acquire them too
        if (!__all_sync(0xffffffffu, f8_wait_chunk(args, tm, abort_flag))) break;
      }
      const int row = tm * F8_BM + row_in_tile;
      const bool row_ok = row < args.M;
      float acc[HN];
#pragma unroll
      for (int j = 0; j < HN; ++j) acc[j] = 0.f;
      bool ok = true;
      auto issue_scales = [&](int k) {
        const uint32_t slot = sring + ((k % F8_SC_RING) * F8_EPI + et) * 8;
        cp_async4(slot, args.sa + (int64_t)k * args.M + (row_ok ? row : 0), row_ok ? 4 : 0);
        cp_async4(slot + 4, args.sb + (int64_t)tn * nkb_b + k, 4);
      };
#pragma unroll 1
      for (int k = 0; k < F8_SC_DIST; ++k) {
        if (k < nk) issue_scales(k);
        cp_async_commit();
      }
      for (int kb = 0; kb < nk; ++kb, ++g) {
        if (kb + F8_SC_DIST < nk) issue_scales(kb + F8_SC_DIST);
        cp_async_commit();
        const uint32_t pb = g % F8_NPB, use = g / F8_NPB;
        ok = bounded_wait(pfull0 + 8 * pb, use & 1, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        tc_fence_after();
        cp_async_wait<F8_SC_DIST>();  // this thread's scales of block kb have landed
        float sa_v, sb_v;
        {
          const uint32_t slot = sring + ((kb % F8_SC_RING) * F8_EPI + et) * 8;
          asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(sa_v), "=f"(sb_v) : "r"(slot));
        }
        const float s = sa_v * sb_v;
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + pb * F8_BN + half * HN;
#pragma unroll
        for (int c = 0; c < HN / 64; ++c) {
          uint32_t r0[32], r1[32];
          tmem_ld32(taddr + c * 64, r0);
          tmem_ld32(taddr + c * 64 + 32, r1);
          tc_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            acc[c * 64 + j] = fmaf(__uint_as_float(r0[j]), s, acc[c * 64 + j]);
            acc[c * 64 + 32 + j] = fmaf(__uint_as_float(r1[j]), s, acc[c * 64 + 32 + j]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(pempty0 + 8 * pb);
      }
      if (!ok) break;
      if (row_ok) {
        __nv_bfloat16* drow;
        if constexpr (REMOTE) {
          const int owner = row / args.rs_rows;
          drow = reinterpret_cast<__nv_bfloat16*>(args.rptrs[owner]) +
                 (int64_t)(args.rs_rank * args.rs_rows + row - owner * args.rs_rows) * args.ldd;
        } else {
          drow = reinterpret_cast<__nv_bfloat16*>(args.D) + (int64_t)row * args.ldd;
        }
#pragma unroll
        for (int v = 0; v < HN / 8; ++v) {
          const int col = tn * F8_BN + half * HN + v * 8;
          if (col >= args.N) break;
          float f[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) f[e] = acc[v * 8 + e];
          if (args.R) {
            const uint4 rv = *reinterpret_cast<const uint4*>(args.R + (int64_t)row * args.ldr + col);
            const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 x = unpack_bf16x2(rw[e]);
              f[2 * e] += x.x;
              f[2 * e + 1] += x.y;
            }
          }
          *reinterpret_cast<uint4*>(drow + col) =
              make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                         pack_bf16x2(f[6], f[7]));
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, F8_NPB * F8_BN);
  }
}

// ------------------------------------------------------------ quantisation
__device__ __forceinline__ uint8_t to_f8(float v, int fmt) {
  __nv_fp8_storage_t r = fmt == 0 ? __nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3)
                                  : __nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E5M2);
  return (uint8_t)r;
}

// Activations / gradients: one warp per (row, 128-wide K block); scale layout [K/128, M].
__global__ void __launch_bounds__(256) quant_1x128_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int M,
                                                          int K, int fmt, float fmax, uint8_t* __restrict__ q,
                                                          int64_t ldq, float* __restrict__ scale) {
  const int lane = threadIdx.x & 31;
  const int64_t w = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
  const int nkb = K / 128;
  if (w >= (int64_t)M * nkb) return;
  const int row = (int)(w / nkb), kb = (int)(w % nkb);
  const uint2 v = *reinterpret_cast<const uint2*>(x + (int64_t)row * ldx + kb * 128 + lane * 4);
  const float2 a = unpack_bf16x2(v.x), b = unpack_bf16x2(v.y);
  float amax = fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(b.x), fabsf(b.y)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float sc = amax > 0.f ? amax / fmax : 1.f;
  const float inv = 1.f / sc;
  const uint32_t packed = (uint32_t)to_f8(a.x * inv, fmt) | ((uint32_t)to_f8(a.y * inv, fmt) << 8) |
                          ((uint32_t)to_f8(b.x * inv, fmt) << 16) | ((uint32_t)to_f8(b.y * inv, fmt) << 24);
  *reinterpret_cast<uint32_t*>(q + (int64_t)row * ldq + kb * 128 + lane * 4) = packed;
  if (lane == 0) scale[(int64_t)kb * M + row] = sc;
}

// Weights: one block per 128 x 128 tile, e4m3; writes W8 [N, K] and, when qt is
// given, W8^T [K, N] (the dgrad operand) with the same block scales.
__global__ void __launch_bounds__(256) quant_128x128_kernel(const __nv_bfloat16* __restrict__ w, int64_t ldw, int N,
                                                            int K, uint8_t* __restrict__ q, uint8_t* __restrict__ qt,
                                                            float* __restrict__ scale) {
  __shared__ float red[8];
  __shared__ uint8_t tile[128][129];
  const int nb = blockIdx.y, kb = blockIdx.x;
  const int nkb = K / 128;
  float amax = 0.f;
  for (int i = threadIdx.x; i < 128 * 128; i += 256) {
    const int r = i / 128, c = i % 128;
    const int n = nb * 128 + r;
    if (n < N) amax = fmaxf(amax, fabsf(__bfloat162float(w[(int64_t)n * ldw + kb * 128 + c])));
  }
  amax = warp_max(amax);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = 0.f;
    for (int k = 0; k < 8; ++k) m = fmaxf(m, red[k]);
    red[0] = m > 0.f ? m / 448.f : 1.f;
    scale[(int64_t)nb * nkb + kb] = red[0];
  }
  __syncthreads();
  const float inv = 1.f / red[0];
  for (int i = threadIdx.x; i < 128 * 128; i += 256) {
    const int r = i / 128, c = i % 128;
    const int n = nb * 128 + r;
    uint8_t v = 0;
    if (n < N) {
      v = to_f8(__bfloat162float(w[(int64_t)n * ldw + kb * 128 + c]) * inv, 0);
      q[(int64_t)n * K + kb * 128 + c] = v;
    }
    tile[r][c] = v;
  }
  if (!qt) return;
  __syncthreads();
  for (int i = threadIdx.x; i < 128 * 128; i += 256) {
    const int c = i / 128, r = i % 128;  // output row = k, column = n
    const int n = nb * 128 + r;
    if (n < N) qt[(int64_t)(kb * 128 + c) * N + n] = tile[r][c];
  }
}

// x = q * scale (1 x 128 blocks, scale layout [K/128, M]) -> bf16
__global__ void __launch_bounds__(256) dequant_1x128_kernel(const uint8_t* __restrict__ q, int M, int K, int fmt,
                                                            const float* __restrict__ scale,
                                                            __nv_bfloat16* __restrict__ x, int64_t ldx) {
  const int64_t n8 = (int64_t)M * K / 8;
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < n8; u += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = u * 8;
    const int row = (int)(e / K), col = (int)(e % K);
    const float sc = scale[(int64_t)(col / 128) * M + row];
    const uint2 v = *reinterpret_cast<const uint2*>(q + e);
    const uint32_t w[2] = {v.x, v.y};
    float f[8];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const __nv_fp8_storage_t bits = (__nv_fp8_storage_t)((w[h] >> (8 * b)) & 0xff);
        const __half_raw hr = __nv_cvt_fp8_to_halfraw(bits, fmt == 0 ? __NV_E4M3 : __NV_E5M2);
        f[h * 4 + b] = __half2float(__half(hr)) * sc;
      }
    *reinterpret_cast<uint4*>(x + (int64_t)row * ldx + col) =
        make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
  }
}

}  // namespace
}  // namespace lk

using namespace lk;

extern "C" int lk_gemm_fp8(const LkGemmFp8Desc* g, cudaStream_t stream) {
  LK_REQUIRE(g->K % 128 == 0 && g->K > 0, "gemm_fp8: K must be a positive multiple of 128");
  LK_REQUIRE(g->N % 8 == 0 && g->a_ld % 16 == 0 && g->b_ld % 16 == 0 && g->ldd % 8 == 0,
             "gemm_fp8: N % 8, operand pitch % 16 bytes, output pitch % 8");
  LK_REQUIRE(g->a_fmt == 0 || g->a_fmt == 1, "gemm_fp8: A format e4m3 (0) or e5m2 (1)");
  if (g->M == 0 || g->N == 0) return 0;
  F8Args a{};
  a.M = g->M;
  a.N = g->N;
  a.K = g->K;
  a.sa = g->sa;
  a.sb = g->sb;
  a.D = g->d;
  a.ldd = g->ldd;
  a.R = reinterpret_cast<const __nv_bfloat16*>(g->r);
  a.ldr = g->ldr;
  a.status = g->status;
  a.tiles_m = cdiv(g->M, F8_BM);
  a.tiles_n = cdiv(g->N, F8_BN);
  CUtensorMap ta, tb;
  const CUtensorMapDataType u8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  if (!make_tmap_2d(&ta, g->a, u8, 1, g->M, g->K, g->a_ld, F8_BM, F8_BK)) return -1;
  if (!make_tmap_2d(&tb, g->b, u8, 1, g->N, g->K, g->b_ld, F8_BN, F8_BK)) return -1;
  a.ag_rows = reinterpret_cast<const uint8_t* const*>(g->ag_rows);
  a.ag_scales = reinterpret_cast<const float* const*>(g->ag_scales);
  a.a_dst = reinterpret_cast<uint8_t*>(const_cast<void*>(g->a));
  a.sa_dst = const_cast<float*>(g->sa);
  a.ag_r = g->ag_rows_per_rank;
  a.ag_rank = g->rank;
  a.ag_world = g->world;
  a.ag_count = g->ag_count;
  a.rptrs = reinterpret_cast<void* const*>(g->rptrs);
  a.rs_rows = g->rs_rows;
  a.rs_rank = g->rank;
  const int grid = std::min(a.tiles_m * a.tiles_n, num_sms());
  const bool ag = g->ag_rows != nullptr, remote = g->rptrs != nullptr;
  if (ag) {
    LK_REQUIRE(g->ag_count && g->ag_scales && g->ag_rows_per_rank % 128 == 0 &&
                   (int64_t)g->ag_rows_per_rank * g->world == g->M && g->a_ld == g->K,
               "gemm_fp8 all-gather: M = world x rows (rows % 128 == 0), dense A");
    if (cudaMemsetAsync(g->ag_count, 0, sizeof(int) * a.tiles_m, stream) != cudaSuccess)
      return fail("gemm_fp8: memset failed");
  }
  if (remote) LK_REQUIRE(g->rs_rows > 0 && g->M % g->rs_rows == 0, "gemm_fp8 reduce-scatter: M = world x rs_rows");
  void* kern = nullptr;
#define LK_F8_PICK(F, AGV, RV) \
  if (g->a_fmt == F && ag == AGV && remote == RV) kern = (void*)gemm_fp8_kernel<F, AGV, RV>;
  LK_F8_PICK(0, false, false) LK_F8_PICK(1, false, false) LK_F8_PICK(0, true, false)
  LK_F8_PICK(0, false, true) LK_F8_PICK(1, true, false) LK_F8_PICK(1, false, true)
#undef LK_F8_PICK
  LK_REQUIRE(kern != nullptr, "gemm_fp8: all-gather and reduce-scatter modes are exclusive");
  static uint64_t attr_set[8] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  const int variant = g->a_fmt * 4 + (ag ? 2 : 0) + (remote ? 1 : 0);
  if (!(attr_set[variant] & (1ull << dev))) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, F8_SMEM);
    attr_set[variant] |= 1ull << dev;
  }
  void* params[] = {&ta, &tb, &a};
  if (ag) {
    // CTAs wait on rows copied by other CTAs: all of them must be resident
    cudaError_t e = cudaLaunchCooperativeKernel(kern, dim3(grid), dim3(F8_THREADS + 64), params, F8_SMEM, stream);
    if (e != cudaSuccess) {
      last_error() = std::string("gemm_fp8 cooperative launch: ") + cudaGetErrorString(e);
      return -1;
    }
  } else {
    cudaError_t e = cudaLaunchKernel(kern, dim3(grid), dim3(F8_THREADS), params, F8_SMEM, stream);
    if (e != cudaSuccess) {
      last_error() = std::string("gemm_fp8 launch: ") + cudaGetErrorString(e);
      return -1;
    }
  }
  return check_launch("gemm_fp8");
}

extern "C" int lk_quant_1x128(const void* x, int64_t ldx, int M, int K, int fmt, void* q, int64_t ldq, float* scale,
                              cudaStream_t s) {
  LK_REQUIRE(K % 128 == 0 && ldx % 4 == 0 && ldq % 4 == 0, "quant_1x128: K % 128, aligned pitches");
  const int64_t warps = (int64_t)M * (K / 128);
  if (warps == 0) return 0;
  quant_1x128_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, s>>>((const __nv_bfloat16*)x, ldx, M, K, fmt,
                                                                  fmt == 0 ? 448.f : 57344.f, (uint8_t*)q, ldq,
                                                                  scale);
  return check_launch("quant_1x128");
}

extern "C" int lk_quant_128x128(const void* w, int64_t ldw, int N, int K, void* q, void* qt, float* scale,
                                cudaStream_t s) {
  LK_REQUIRE(K % 128 == 0 && N % 16 == 0, "quant_128x128: K % 128, N % 16");
  dim3 grid(K / 128, (N + 127) / 128);
  quant_128x128_kernel<<<grid, 256, 0, s>>>((const __nv_bfloat16*)w, ldw, N, K, (uint8_t*)q, (uint8_t*)qt, scale);
  return check_launch("quant_128x128");
}

extern "C" int lk_dequant_1x128(const void* q, int M, int K, int fmt, const float* scale, void* x, int64_t ldx,
                                cudaStream_t s) {
  LK_REQUIRE(K % 128 == 0 && ldx % 8 == 0, "dequant_1x128: K % 128, ldx % 8");
  const int64_t n8 = (int64_t)M * K / 8;
  if (n8 == 0) return 0;
  const int grid = (int)std::min<int64_t>((n8 + 255) / 256, 8 * num_sms());
  dequant_1x128_kernel<<<grid, 256, 0, s>>>((const uint8_t*)q, M, K, fmt, scale, (__nv_bfloat16*)x, ldx);
  return check_launch("dequant_1x128");
}
