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
// writes an fp32 partial [split, M, N] and a reduction kernel sums them in
// split order (deterministic, so a CUDA-graph replay equals an eager step).
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
constexpr int DQ_THREADS = 96 + 32 * DQ_CONV_WARPS;  // raw TMA, MMA, X TMA, converters

// Ring sizes.  The raw weight ring is decoupled from the dequantised-tile ring
// and is as deep as the shared-memory budget allows: the weights are the HBM
// stream, so its loads run up to RAW_STAGES stages ahead of the converters.
// The activation ring is deeper for small batches (its tiles come from L2).
// Up to MP = 128 two CTAs stay resident per SM.
template <int FMT, int MP>
struct DqCfg {
  static constexpr int RAW_ROW = FMT == 2 ? DQ_BK / 2 : DQ_BK;  // raw bytes per weight row per stage
  static constexpr int RAW_TILE = DQ_BM * RAW_ROW;
  static constexpr int A_BYTES = DQ_BM * DQ_BK * 2;  // dequantised bf16 tile
  static constexpr int A_STAGES = 2;
  static constexpr int X_BYTES = MP * DQ_BK * 2;
  static constexpr int X_STAGES = MP <= 16 ? 8 : (MP <= 32 ? 6 : (MP <= 64 ? 4 : 3));
  static constexpr int BUDGET = (MP <= 128 ? 104 : 200) * 1024;
  static constexpr int RAW_LEFT = (BUDGET - A_STAGES * A_BYTES - X_STAGES * X_BYTES) / RAW_TILE;
  static constexpr int RAW_STAGES = RAW_LEFT > 12 ? 12 : RAW_LEFT;
  static_assert(RAW_STAGES >= 2, "dq_gemm: raw ring too shallow");
  static constexpr int NBAR = 2 * (RAW_STAGES + A_STAGES + X_STAGES) + 2;
  static constexpr int SMEM =
      A_STAGES * A_BYTES + X_STAGES * X_BYTES + RAW_STAGES * RAW_TILE + NBAR * 8 + 16 + 1024;
  static constexpr int TMEM_COLS = MP < 32 ? 32 : MP;
  static constexpr int MIN_BLOCKS = MP <= 128 ? 2 : 1;
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

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// (a & 0x000F000F) | 0x43004300: two 4-bit codes into the low mantissa bits of
// a bf16 pair with exponent 2^7, i.e. the exact values 128 + q.
__device__ __forceinline__ uint32_t nib_to_bf16x2(uint32_t a) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(0x000F000Fu), "r"(0x43004300u));
  return d;
}

__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
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

// The same in bf16x2 arithmetic, for zero points z in [-241, 128]: byte permutes
// put codes 2i and 2i+1 into one word, 128 + q is formed exactly in the
// mantissa, (128 + q) - (128 + z) = q - z is exact (|q - z| <= 256), and one
// rounding multiply by s (s rounded to bf16) gives the value.
// zz = bf16x2(128 + z), ss = bf16x2(s).
__device__ __forceinline__ uint4 dq_int4x8_fast(uint32_t v, uint32_t zz, uint32_t ss) {
  const uint32_t hi = v >> 4;
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    // byte 0 <- byte i of v (code 2i in its low nibble), byte 2 <- byte i of v >> 4 (code 2i + 1)
    const uint32_t w = nib_to_bf16x2(prmt(v, hi, 0x0400u + 0x0101u * (uint32_t)i));
    o[i] = bf16x2_mul(bf16x2_sub(w, zz), ss);
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

__device__ __forceinline__ void conv_bar_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(32 * DQ_CONV_WARPS) : "memory");
}

// Wait for every load issued into a ring whose slots are flagged in `pending`
// (slot i at parity bit i of `par`), so no copy lands after the CTA exits.
__device__ __forceinline__ void drain_ring(uint32_t full0, uint32_t pending, uint32_t par, int stages,
                                           int* status) {
  for (int i = 0; i < stages; ++i)
    if (pending & (1u << i)) bounded_wait(full0 + 8 * i, (par >> i) & 1, status, LK_ERR_TIMEOUT_DRAIN, nullptr);
}

template <int FMT, int MP>
__global__ void __launch_bounds__(DQ_THREADS, (DqCfg<FMT, MP>::MIN_BLOCKS))
    dq_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                   const DqArgs args) {
  using C = DqCfg<FMT, MP>;
  constexpr int RS = C::RAW_STAGES, AS = C::A_STAGES, XS = C::X_STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const uint32_t sA = smem_u32(smem);              // AS x 16 KB dequantised tiles
  const uint32_t sX = sA + AS * C::A_BYTES;        // XS x X tiles
  const uint32_t sR = sX + XS * C::X_BYTES;        // RS x raw weight tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + AS * C::A_BYTES + XS * C::X_BYTES + RS * C::RAW_TILE);
  const uint32_t rfull0 = smem_u32(bars);
  const uint32_t rempty0 = rfull0 + 8 * RS;
  const uint32_t afull0 = rempty0 + 8 * RS;
  const uint32_t aempty0 = afull0 + 8 * AS;
  const uint32_t xfull0 = aempty0 + 8 * AS;
  const uint32_t xempty0 = xfull0 + 8 * XS;
  const uint32_t accfull = xempty0 + 8 * XS;
  const uint32_t drain_bar = accfull + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int n0 = blockIdx.x * DQ_BM;
  const int k_begin = blockIdx.y * args.k_split;
  const int nk = min(args.k_split, args.K - k_begin) / DQ_BK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < RS; ++i) {
      mbar_init(rfull0 + 8 * i, 1);
      mbar_init(rempty0 + 8 * i, DQ_CONV_WARPS);
    }
    for (int i = 0; i < AS; ++i) {
      mbar_init(afull0 + 8 * i, DQ_CONV_WARPS);
      mbar_init(aempty0 + 8 * i, 1);
    }
    for (int i = 0; i < XS; ++i) {
      mbar_init(xfull0 + 8 * i, 1);
      mbar_init(xempty0 + 8 * i, 1);
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
    // ------------------------------------------------------- raw weight TMA
    if (lane == 0) {
      uint32_t pending = 0, par = 0;
      for (int kb = 0; kb < nk; ++kb) {
        const int r = kb % RS;
        const uint32_t ph = (uint32_t)(kb / RS) & 1;
        if (!bounded_wait(rempty0 + 8 * r, ph ^ 1, args.status, LK_ERR_TIMEOUT_EMPTY, abort_flag)) {
          drain_ring(rfull0, pending, par, RS, args.status);
          break;
        }
        const int k0 = k_begin + kb * DQ_BK;
        mbar_expect_tx(rfull0 + 8 * r, C::RAW_TILE);
        tma_load_2d(sR + r * C::RAW_TILE, &tmW, rfull0 + 8 * r, FMT == 2 ? k0 / 2 : k0, n0);
        pending |= 1u << r;
        par = (par & ~(1u << r)) | (ph << r);
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------------- activation TMA
    if (lane == 0) {
      uint32_t pending = 0, par = 0;
      for (int kb = 0; kb < nk; ++kb) {
        const int x = kb % XS;
        const uint32_t ph = (uint32_t)(kb / XS) & 1;
        if (!bounded_wait(xempty0 + 8 * x, ph ^ 1, args.status, LK_ERR_TIMEOUT_EMPTY, abort_flag)) {
          drain_ring(xfull0, pending, par, XS, args.status);
          break;
        }
        mbar_expect_tx(xfull0 + 8 * x, C::X_BYTES);
        tma_load_2d(sX + x * C::X_BYTES, &tmX, xfull0 + 8 * x, k_begin + kb * DQ_BK, 0);
        pending |= 1u << x;
        par = (par & ~(1u << x)) | (ph << x);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(DQ_BM, MP, false, false);
      bool ok = true;
      for (int kb = 0; kb < nk && ok; ++kb) {
        const int s = kb % AS, x = kb % XS;
        ok = bounded_wait(afull0 + 8 * s, (uint32_t)(kb / AS) & 1, args.status, LK_ERR_TIMEOUT_FULL, abort_flag) &&
             bounded_wait(xfull0 + 8 * x, (uint32_t)(kb / XS) & 1, args.status, LK_ERR_TIMEOUT_FULL, abort_flag);
        if (!ok) break;
        tc_fence_after();
        const uint32_t a = sA + s * C::A_BYTES, xb = sX + x * C::X_BYTES;
#pragma unroll
        for (int kk = 0; kk < DQ_BK / 16; ++kk)
          tc_mma_f16(tmem, make_desc_sw128(a + kk * 32, 16, 1024), make_desc_sw128(xb + kk * 32, 16, 1024), idesc,
                     (kb | kk) != 0 ? 1u : 0u);
        tc_commit(aempty0 + 8 * s);
        tc_commit(xempty0 + 8 * x);
      }
      if (ok) tc_commit(accfull);
      tc_commit(drain_bar);
      bounded_wait(drain_bar, 0, args.status, LK_ERR_TIMEOUT_DRAIN, nullptr);
    }
  } else {
    // ------------------------------------------------------- converters
    const int t = threadIdx.x - 96;
    const int r = t & (DQ_BM - 1);  // weight row within the tile
    const int h = t >> 7;           // which 32 of the stage's 64 K values
    const int n = n0 + r;
    const bool row_ok = n < args.N;
    const int groups = FMT == 2 ? args.K / args.group : 1;
    float s_cur = 0.f, z_cur = 0.f, s_nxt = 0.f, z_nxt = 0.f;
    if (row_ok) {
      if constexpr (FMT == 2) {
        const int64_t gi = (int64_t)n * groups + (k_begin + h * 32) / args.group;
        s_nxt = args.scale[gi];
        z_nxt = args.zero[gi];
      } else {
        s_nxt = args.scale[n];
      }
    }
    bool ok = true;
    for (int kb = 0; kb < nk; ++kb) {
      const int rs = kb % RS, s = kb % AS;
      s_cur = s_nxt;
      z_cur = z_nxt;
      if constexpr (FMT == 2) {
        // next stage's group scale and zero point, loaded a stage ahead
        if (row_ok && kb + 1 < nk) {
          const int64_t gi = (int64_t)n * groups + (k_begin + (kb + 1) * DQ_BK + h * 32) / args.group;
          s_nxt = args.scale[gi];
          z_nxt = args.zero[gi];
        }
      }
      ok = bounded_wait(rfull0 + 8 * rs, (uint32_t)(kb / RS) & 1, args.status, LK_ERR_TIMEOUT_FULL, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      const uint8_t* raw = smem + (sR - sA) + rs * C::RAW_TILE + r * C::RAW_ROW;
      uint32_t w[FMT == 2 ? 4 : 8];
      if constexpr (FMT == 2) {
        const uint4 v = *reinterpret_cast<const uint4*>(raw + h * 16);
        w[0] = v.x, w[1] = v.y, w[2] = v.z, w[3] = v.w;
      } else {
        const uint4 v0 = *reinterpret_cast<const uint4*>(raw + h * 32);
        const uint4 v1 = *reinterpret_cast<const uint4*>(raw + h * 32 + 16);
        w[0] = v0.x, w[1] = v0.y, w[2] = v0.z, w[3] = v0.w, w[4] = v1.x, w[5] = v1.y, w[6] = v1.z, w[7] = v1.w;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(rempty0 + 8 * rs);  // the raw slot may be refilled
      ok = bounded_wait(aempty0 + 8 * s, ((uint32_t)(kb / AS) & 1) ^ 1, args.status, LK_ERR_TIMEOUT_EMPTY,
                        abort_flag);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      uint8_t* a_tile = smem + s * C::A_BYTES;
      if constexpr (FMT == 2) {
        if (z_cur >= -241.f && z_cur <= 128.f) {
          const uint32_t zz = pack_bf16x2(128.f + z_cur, 128.f + z_cur);
          const uint32_t ss = pack_bf16x2(s_cur, s_cur);
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint4 o = row_ok ? dq_int4x8_fast(w[c], zz, ss) : make_uint4(0u, 0u, 0u, 0u);
            *reinterpret_cast<uint4*>(a_tile + dq_sw128(r, h * 4 + c)) = o;
          }
        } else {
          const float zs = z_cur * s_cur;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint4 o = row_ok ? dq_int4x8(w[c], s_cur, zs) : make_uint4(0u, 0u, 0u, 0u);
            *reinterpret_cast<uint4*>(a_tile + dq_sw128(r, h * 4 + c)) = o;
          }
        }
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint4 o = row_ok ? dq_byte8<FMT>(w[2 * c], w[2 * c + 1], s_cur) : make_uint4(0u, 0u, 0u, 0u);
          *reinterpret_cast<uint4*>(a_tile + dq_sw128(r, h * 4 + c)) = o;
        }
      }
      fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core's async reads
      __syncwarp();
      if (lane == 0) mbar_arrive(afull0 + 8 * s);
    }
    // -------------------------------------------------------- epilogue
    const bool split = gridDim.y > 1;
    if (warp < 7) {  // warps 3..6: one per TMEM lane quarter
      const int q = warp & 3;
      const int nrow = n0 + q * 32 + lane;
      ok = ok && bounded_wait(accfull, 0, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag);
      if (__all_sync(0xffffffffu, ok)) {
        tc_fence_after();
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16);
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
    if (split && args.counters) {
      // Split-K: the last split of this weight tile to finish sums all the
      // partials in split order (deterministic) and writes Y (+ R).
      conv_bar_sync();  // this CTA's partial stores precede the release below
      if (t == 0) {
        __threadfence();
        const int prev = atomicAdd(args.counters + blockIdx.x, 1);
        *last_flag = prev == (int)gridDim.y - 1;
      }
      conv_bar_sync();
      if (*last_flag) {
        __threadfence();
        const int nn = n0 + r;
        if (nn < args.N) {
          for (int m = h; m < args.M; m += 2) {
            float acc = 0.f;
            for (int sp = 0; sp < (int)gridDim.y; ++sp)
              acc += __ldcg(args.partial + ((int64_t)sp * args.M + m) * args.N + nn);
            if (args.r) acc += __bfloat162float(args.r[(int64_t)m * args.ldr + nn]);
            args.y[(int64_t)m * args.ldy + nn] = __float2bfloat16(acc);
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
  using C = DqCfg<FMT, MP>;
  CUtensorMap tw, tx;
  if (!make_tmap_2d(&tw, d.q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, d.N, FMT == 2 ? d.K / 2 : d.K,
                    FMT == 2 ? d.K / 2 : d.K, DQ_BM, C::RAW_ROW, CU_TENSOR_MAP_SWIZZLE_NONE))
    return -1;
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
  a.counters = splits > 1 ? d.counters : nullptr;
  a.status = d.status;
  auto k = dq_gemm_kernel<FMT, MP>;
  static uint64_t attr_set = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set & (1ull << dev))) {
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    attr_set |= 1ull << dev;
  }
  dim3 grid(cdiv(d.N, DQ_BM), splits);
  k<<<grid, DQ_THREADS, C::SMEM, s>>>(tw, tx, a);
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
  // Split K until the grid fills the resident CTA slots (two per SM up to 128
  // batch rows) without a second partial wave; every split keeps at least 4 K
  // stages, and the fp32 partials (written and read back once) stay within
  // about twice the int4 weight bytes.
  const int tiles = cdiv(N, DQ_BM);
  const int slots = (M <= 128 ? 2 : 1) * num_sms();
  int splits = std::max(1, slots / tiles);
  splits = std::min(splits, std::max(1, K / (4 * DQ_BK)));
  splits = std::min(splits, std::max(1, K / (8 * std::max(M, 1))));
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
