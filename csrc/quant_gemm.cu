// K14, decode form: weight-streaming dequant GEMM on the 5th-generation tensor cores.
//
//   Y[M, N] (bf16) = X[M, K] (bf16) . dequant(W)[N, K]^T  (+ R[M, N])
//
// for the decode batches of serving (M <= 256 rows), where the weights are the
// bytes that matter: int4 (group-wise scale and zero point, two values per
// byte, low nibble first), int8 or fp8 e4m3 (one scale per row).  The weight
// tile is the MMA's A operand (128 weight rows) and the activations its N
// operand (M padded to MP = 16 ... 256), so one pass over the weights serves the
// whole batch: D^T[n, m] accumulates in TMEM (128 lanes x MP columns).
//
// Per CTA: 128 weight rows x a K range (split-K over blockIdx.y), 64-wide K
// stages in a ring:
//   warp 0      TMA: the stage's raw weight tile (no swizzle) and X tile
//               (128B swizzle; rows >= M read as zeros);
//   warp 1      TMEM owner; one thread issues tcgen05.mma.kind::f16 (M 128,
//               N MP, K 16) x 4 per stage and commits the stage back;
//   warps 2..9  converters: dequantise the raw tile into bf16 in the 128B-swizzled
//               K-major layout the MMA reads (thread = weight row x 32 K values),
//               fence the generic-proxy stores for the async proxy, arrive; then
//               warps 2..5 (one per TMEM lane quarter) drain the accumulator:
//               thread = weight row, one coalesced store per batch row.
// With one split the epilogue writes bf16 Y (+ R); with several, each split
// writes an fp32 partial [split, M, N] and the partials are summed in split
// order (deterministic, so a CUDA-graph replay equals an eager step): for
// batches up to 4 rows by the last split of each weight tile to finish (tile
// counters, same launch), else by a second, grid-wide kernel.
// Every wait is bounded.
//
// Reference: QuantizedInferenceKernels (include/api/serving_production.hpp:211-226)
// and the INT4 quantizer's dequantisation (include/nn/quantization_production.hpp:190-221)
// run on the CPU with one scale per tensor; this is the tensor-core form.
#include "common.cuh"
#include "host_util.h"
#include "lk_api.h"

namespace lk {
namespace {

constexpr int DQ_BM = 128, DQ_BK = 64;
constexpr int DQ_CONV_WARPS = 8;
constexpr int DQ_THREADS = 64 + 32 * DQ_CONV_WARPS;

template <int FMT>  // 0 int8, 1 fp8 e4m3, 2 int4
struct DqRaw {
  static constexpr int ROW_BYTES = FMT == 2 ? DQ_BK / 2 : DQ_BK;  // raw bytes per weight row per stage
  static constexpr int TILE = DQ_BM * ROW_BYTES;
};

// Stage counts keep two CTAs resident per SM (up to MP = 128), so one CTA's
// pipeline fill and epilogue overlap the other's stream of weights.
template <int MP>
struct DqCfg {
  static constexpr int STAGES = MP >= 256 ? 2 : (MP >= 64 ? 3 : 4);
  static constexpr int A_BYTES = DQ_BM * DQ_BK * 2;  // dequantised bf16 tile
  static constexpr int X_BYTES = MP * DQ_BK * 2;
  static constexpr int TMEM_COLS = MP < 32 ? 32 : MP;
};

struct DqArgs {
  int M, N, K, group;
  int k_split;  // K elements per split (multiple of 64)
  const float* scale;  // int4: [N, K / group]; int8 / fp8: [N]
  const float* zero;   // int4: [N, K / group]
  __nv_bfloat16* y;
  int64_t ldy;
  const __nv_bfloat16* r;  // optional residual [M, N]
  int64_t ldr;
  float* partial;  // [splits, M, N] when gridDim.y > 1
  int* counters;   // per weight tile, zero between launches: the last split to finish reduces
  int* status;
};

__device__ __forceinline__ uint32_t dq_sw128(int row, int chunk) {
  return (uint32_t)(row * 128 + (((chunk ^ (row & 7)) & 7) << 4));
}

// 8 int4 values (one 32-bit word, low nibble first) -> 8 floats (q - z) * s, as 4 bf16 pairs
__device__ __forceinline__ uint4 dq_int4x8(uint32_t v, float s, float zs) {
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    // exact integer -> float through the mantissa of 2^23: (2^23 + q) - 2^23
    const float a = __uint_as_float(0x4B000000u | ((v >> (8 * i)) & 0xFu)) - 8388608.f;
    const float b = __uint_as_float(0x4B000000u | ((v >> (8 * i + 4)) & 0xFu)) - 8388608.f;
    o[i] = pack_bf16x2(fmaf(a, s, -zs), fmaf(b, s, -zs));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// 8 int8 / fp8 values (two 32-bit words) -> bf16 x 8, times s
template <int FMT>
__device__ __forceinline__ uint4 dq_byte8(uint32_t lo, uint32_t hi, float s) {
  const uint32_t w[2] = {lo, hi};
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t word = w[i >> 1];
    const int sh = (i & 1) * 16;
    float a, b;
    if constexpr (FMT == 0) {
      a = (float)(int8_t)((word >> sh) & 0xFFu);
      b = (float)(int8_t)((word >> (sh + 8)) & 0xFFu);
    } else {
      a = __half2float(__half(__nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)((word >> sh) & 0xFFu), __NV_E4M3)));
      b = __half2float(__half(__nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)((word >> (sh + 8)) & 0xFFu), __NV_E4M3)));
    }
    o[i] = pack_bf16x2(a * s, b * s);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

template <int FMT, int MP>
__global__ void __launch_bounds__(DQ_THREADS, 2)
    dq_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                   const DqArgs args) {
  using C = DqCfg<MP>;
  using RW = DqRaw<FMT>;
  constexpr int S = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const uint32_t sA = smem_u32(smem);                  // S x 16 KB dequantised tiles
  const uint32_t sX = sA + S * C::A_BYTES;             // S x X tiles
  const uint32_t sR = sX + S * C::X_BYTES;             // S x raw weight tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * (C::A_BYTES + C::X_BYTES + RW::TILE));
  const uint32_t rawfull0 = smem_u32(bars);
  const uint32_t full0 = rawfull0 + 8 * S;
  const uint32_t empty0 = full0 + 8 * S;
  const uint32_t accfull = empty0 + 8 * S;
  const uint32_t drain_bar = accfull + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * S + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int n0 = blockIdx.x * DQ_BM;
  const int k_begin = blockIdx.y * args.k_split;
  const int nk = min(args.k_split, args.K - k_begin) / DQ_BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(rawfull0 + 8 * s, 1);
      mbar_init(full0 + 8 * s, 1 + DQ_CONV_WARPS);
      mbar_init(empty0 + 8 * s, 1);
    }
    mbar_init(accfull, 1);
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    *last_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA
    if (lane == 0) {
      uint32_t pending = 0, parbits = 0;
      bool ok = true;
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % S;
        const uint32_t ph = (uint32_t)(kb / S) & 1;
        if (!bounded_wait(empty0 + 8 * s, ph ^ 1, args.status, LK_ERR_TIMEOUT_EMPTY, abort_flag)) {
          ok = false;
          break;
        }
        const int k0 = k_begin + kb * DQ_BK;
        mbar_expect_tx(rawfull0 + 8 * s, RW::TILE);
        tma_load_2d(sR + s * RW::TILE, &tmW, rawfull0 + 8 * s, FMT == 2 ? k0 / 2 : k0, n0);
        mbar_expect_tx(full0 + 8 * s, C::X_BYTES);
        tma_load_2d(sX + s * C::X_BYTES, &tmX, full0 + 8 * s, k0, 0);
        pending |= 1u << s;
        parbits = (parbits & ~(1u << s)) | (ph << s);
      }
      if (!ok)
        for (int i = 0; i < S; ++i)
          if (pending & (1u << i)) {
            bounded_wait(rawfull0 + 8 * i, (parbits >> i) & 1, args.status, LK_ERR_TIMEOUT_DRAIN, nullptr);
          }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(DQ_BM, MP, false, false);
      bool ok = true;
      for (int kb = 0; kb < nk && ok; ++kb) {
        const int s = kb % S;
        if (!bounded_wait(full0 + 8 * s, (uint32_t)(kb / S) & 1, args.status, LK_ERR_TIMEOUT_FULL, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a = sA + s * C::A_BYTES, x = sX + s * C::X_BYTES;
#pragma unroll
        for (int kk = 0; kk < DQ_BK / 16; ++kk)
          tc_mma_f16(tmem, make_desc_sw128(a + kk * 32, 16, 1024), make_desc_sw128(x + kk * 32, 16, 1024), idesc,
                     (kb | kk) != 0 ? 1u : 0u);
        tc_commit(empty0 + 8 * s);
      }
      if (ok) tc_commit(accfull);
      tc_commit(drain_bar);
      bounded_wait(drain_bar, 0, args.status, LK_ERR_TIMEOUT_DRAIN, nullptr);
    }
  } else {
    // ------------------------------------------------------- converters
    const int t = threadIdx.x - 64;
    const int r = t & (DQ_BM - 1);  // weight row within the tile
    const int h = t >> 7;           // which 32 of the stage's 64 K values
    const int n = n0 + r;
    const bool row_ok = n < args.N;
    const int groups = FMT == 2 ? args.K / args.group : 1;
    float s_cur = 0.f, z_cur = 0.f;
    if (FMT != 2 && row_ok) s_cur = args.scale[n];
    bool ok = true;
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % S;
      const int k0 = k_begin + kb * DQ_BK + h * 32;
      if constexpr (FMT == 2) {
        if (row_ok) {
          const int g = k0 / args.group;
          s_cur = args.scale[(int64_t)n * groups + g];
          z_cur = args.zero[(int64_t)n * groups + g];
        }
      }
      ok = bounded_wait(rawfull0 + 8 * s, (uint32_t)(kb / S) & 1, args.status, LK_ERR_TIMEOUT_FULL, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      const uint8_t* raw = smem + (sR - sA) + s * RW::TILE + r * RW::ROW_BYTES;
      uint8_t* a_tile = smem + s * C::A_BYTES;
      if constexpr (FMT == 2) {
        const uint4 v = row_ok ? *reinterpret_cast<const uint4*>(raw + h * 16) : make_uint4(0u, 0u, 0u, 0u);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        const float zs = z_cur * s_cur;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint4 o = row_ok ? dq_int4x8(w[c], s_cur, zs) : make_uint4(0u, 0u, 0u, 0u);
          *reinterpret_cast<uint4*>(a_tile + dq_sw128(r, h * 4 + c)) = o;
        }
      } else {
        const uint4 v0 = row_ok ? *reinterpret_cast<const uint4*>(raw + h * 32) : make_uint4(0u, 0u, 0u, 0u);
        const uint4 v1 = row_ok ? *reinterpret_cast<const uint4*>(raw + h * 32 + 16) : make_uint4(0u, 0u, 0u, 0u);
        const uint32_t w[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint4 o = row_ok ? dq_byte8<FMT>(w[2 * c], w[2 * c + 1], s_cur) : make_uint4(0u, 0u, 0u, 0u);
          *reinterpret_cast<uint4*>(a_tile + dq_sw128(r, h * 4 + c)) = o;
        }
      }
      fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core's async reads
      __syncwarp();
      if (lane == 0) mbar_arrive(full0 + 8 * s);
    }
    // -------------------------------------------------------- epilogue
    if (warp < 6) {
      const int q = warp & 3;  // TMEM lane quarter
      const int nrow = n0 + q * 32 + lane;
      ok = ok && bounded_wait(accfull, 0, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag);
      if (__all_sync(0xffffffffu, ok)) {
        tc_fence_after();
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16);
        const bool split = gridDim.y > 1;
#pragma unroll 1
        for (int c = 0; c < MP; c += (MP < 32 ? 16 : 32)) {
          float v[32];
          if constexpr (MP < 32) {
            uint32_t rr[16];
            tmem_ld16(taddr + c, rr);
            tc_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(rr[j]);
          } else {
            uint32_t rr[32];
            tmem_ld32(taddr + c, rr);
            tc_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(rr[j]);
          }
          if (nrow < args.N) {
#pragma unroll
            for (int j = 0; j < (MP < 32 ? 16 : 32); ++j) {
              const int m = c + j;
              if (m >= args.M) break;
              if (split) {
                args.partial[((int64_t)blockIdx.y * args.M + m) * args.N + nrow] = v[j];
              } else {
                float o = v[j];
                if (args.r) o += __bfloat162float(args.r[(int64_t)m * args.ldr + nrow]);
                args.y[(int64_t)m * args.ldy + nrow] = __float2bfloat16(o);
              }
            }
          }
        }
      }
    }
    if (gridDim.y > 1 && args.counters) {
      // Split-K: the last split of this weight tile to finish sums all the
      // partials in split order (deterministic) and writes Y (+ R).
      asm volatile("bar.sync 1, %0;" ::"n"(32 * DQ_CONV_WARPS) : "memory");  // partial stores first
      if (t == 0) {
        __threadfence();
        const int prev = atomicAdd(args.counters + blockIdx.x, 1);
        *last_flag = prev == (int)gridDim.y - 1;
      }
      asm volatile("bar.sync 1, %0;" ::"n"(32 * DQ_CONV_WARPS) : "memory");
      if (*last_flag) {
        __threadfence();
        if (n < args.N) {
          for (int m = h; m < args.M; m += 2) {
            float acc = 0.f;
            for (int sp = 0; sp < (int)gridDim.y; ++sp)
              acc += __ldcg(args.partial + ((int64_t)sp * args.M + m) * args.N + n);
            if (args.r) acc += __bfloat162float(args.r[(int64_t)m * args.ldr + n]);
            args.y[(int64_t)m * args.ldy + n] = __float2bfloat16(acc);
          }
        }
        if (t == 0) args.counters[blockIdx.x] = 0;  // ready for the next launch
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// Y = sum over splits of the fp32 partials (in split order) (+ R), as bf16.
__global__ void dq_reduce_kernel(const float* __restrict__ partial, int splits, int M, int N,
                                 const __nv_bfloat16* __restrict__ r, int64_t ldr, __nv_bfloat16* __restrict__ y,
                                 int64_t ldy) {
  const int64_t total = (int64_t)M * N / 4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = i * 4;
    const int m = (int)(e / N), n = (int)(e % N);
    float4 acc = *reinterpret_cast<const float4*>(partial + e);
    for (int sp = 1; sp < splits; ++sp) {
      const float4 p = *reinterpret_cast<const float4*>(partial + (int64_t)sp * M * N + e);
      acc.x += p.x;
      acc.y += p.y;
      acc.z += p.z;
      acc.w += p.w;
    }
    if (r) {
      const uint2 rv = *reinterpret_cast<const uint2*>(r + (int64_t)m * ldr + n);
      const float2 a = unpack_bf16x2(rv.x), b = unpack_bf16x2(rv.y);
      acc.x += a.x;
      acc.y += a.y;
      acc.z += b.x;
      acc.w += b.y;
    }
    *reinterpret_cast<uint2*>(y + (int64_t)m * ldy + n) = make_uint2(pack_bf16x2(acc.x, acc.y), pack_bf16x2(acc.z, acc.w));
  }
}

template <int FMT, int MP>
int launch_dq(const LkDqGemmDesc& d, int splits, int k_split, cudaStream_t s) {
  using C = DqCfg<MP>;
  using RW = DqRaw<FMT>;
  CUtensorMap tw, tx;
  if (FMT == 2) {
    if (!make_tmap_2d(&tw, d.q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, d.N, d.K / 2, d.K / 2, DQ_BM, RW::ROW_BYTES,
                      CU_TENSOR_MAP_SWIZZLE_NONE))
      return -1;
  } else if (!make_tmap_2d(&tw, d.q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, d.N, d.K, d.K, DQ_BM, RW::ROW_BYTES,
                           CU_TENSOR_MAP_SWIZZLE_NONE)) {
    return -1;
  }
  if (!make_tmap_2d(&tx, d.x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, d.M, d.K, d.ldx, MP, DQ_BK)) return -1;
  DqArgs a{};
  a.M = d.M;
  a.N = d.N;
  a.K = d.K;
  a.group = d.group;
  a.k_split = k_split;
  a.scale = d.scale;
  a.zero = d.zero;
  a.y = (__nv_bfloat16*)d.y;
  a.ldy = d.ldy;
  a.r = (const __nv_bfloat16*)d.r;
  a.ldr = d.ldr;
  a.partial = d.partial;
  // the in-kernel reduction runs on one CTA per weight tile, so it only pays while
  // the partials are few (measured: a gain at 1 row, a loss from 16); larger
  // batches use the grid-wide reduction kernel
  a.counters = (splits > 1 && d.M <= 4) ? d.counters : nullptr;
  a.status = d.status;
  constexpr int SMEM = C::STAGES * (C::A_BYTES + C::X_BYTES + RW::TILE) + 3 * C::STAGES * 8 + 64 + 1024;
  auto k = dq_gemm_kernel<FMT, MP>;
  static uint64_t attr_set = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set & (1ull << dev))) {
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    attr_set |= 1ull << dev;
  }
  dim3 grid(cdiv(d.N, DQ_BM), splits);
  k<<<grid, DQ_THREADS, SMEM, s>>>(tw, tx, a);
  if (check_launch("dq_gemm")) return -1;
  if (splits > 1 && !a.counters) {
    const int64_t n4 = (int64_t)d.M * d.N / 4;
    const int g = (int)std::min<int64_t>((n4 + 255) / 256, (int64_t)num_sms() * 8);
    dq_reduce_kernel<<<g, 256, 0, s>>>(d.partial, splits, d.M, d.N, (const __nv_bfloat16*)d.r, d.ldr,
                                       (__nv_bfloat16*)d.y, d.ldy);
    return check_launch("dq_reduce");
  }
  return 0;
}

template <int FMT>
int launch_dq_fmt(const LkDqGemmDesc& d, int splits, int k_split, cudaStream_t s) {
  if (d.M <= 16) return launch_dq<FMT, 16>(d, splits, k_split, s);
  if (d.M <= 32) return launch_dq<FMT, 32>(d, splits, k_split, s);
  if (d.M <= 64) return launch_dq<FMT, 64>(d, splits, k_split, s);
  if (d.M <= 128) return launch_dq<FMT, 128>(d, splits, k_split, s);
  return launch_dq<FMT, 256>(d, splits, k_split, s);
}

}  // namespace
}  // namespace lk

using namespace lk;

extern "C" int lk_dq_gemm_splits(int M, int N, int K) {
  // Split K until the grid fills the two resident CTA slots per SM without a
  // second, partial wave; every split keeps at least 4 K stages.
  const int tiles = cdiv(N, DQ_BM);
  int splits = std::max(1, 2 * num_sms() / tiles);
  splits = std::min(splits, std::max(1, K / (4 * DQ_BK)));
  (void)M;
  return splits;
}

extern "C" int lk_dq_gemm(const LkDqGemmDesc* d, cudaStream_t s) {
  LK_REQUIRE(d->M >= 1 && d->M <= 256, "dq_gemm: 1 <= M <= 256 (decode batches)");
  LK_REQUIRE(d->K % DQ_BK == 0 && d->N % 4 == 0, "dq_gemm: K % 64 == 0, N % 4 == 0");
  LK_REQUIRE(d->ldx % 8 == 0 && d->ldy % 4 == 0 && (!d->r || d->ldr % 4 == 0), "dq_gemm: pitches");
  LK_REQUIRE(d->fmt != LK_Q_INT4 || (d->group % DQ_BK == 0 && d->K % d->group == 0 && d->zero),
             "dq_gemm: int4 groups must be multiples of 64 dividing K");
  int splits = d->splits > 0 ? d->splits : lk_dq_gemm_splits(d->M, d->N, d->K);
  int k_split = cdiv(d->K, (int64_t)splits * DQ_BK) * DQ_BK;
  splits = cdiv(d->K, k_split);
  LK_REQUIRE(splits == 1 || d->partial, "dq_gemm: split-K needs the fp32 partial buffer [splits, M, N]");
  LK_REQUIRE(splits == 1 || !d->counters || cdiv(d->N, DQ_BM) <= LK_DQ_COUNTERS,
             "dq_gemm: more weight tiles than split-K counters");
  if (d->fmt == LK_Q_INT4) return launch_dq_fmt<2>(*d, splits, k_split, s);
  if (d->fmt == LK_Q_FP8) return launch_dq_fmt<1>(*d, splits, k_split, s);
  if (d->fmt == LK_Q_INT8) return launch_dq_fmt<0>(*d, splits, k_split, s);
  return fail("dq_gemm: unknown format");
}
