// K2, MX form: fp8 GEMM with hardware block scaling on the 5th-generation tensor cores.
//
//   D[m, n] = sum_k 2^ea[m, k/32] * 2^eb[n, k/32] * A8[m, k] * B8[n, k]   (+ R[m, n])
//
// A8 [M, K] and B8 [N, K] hold fp8 bits (A e4m3 or e5m2, B e4m3 or e5m2), K-major.
// The scales are UE8M0 exponents (one byte, value 2^(byte - 127)) per row and
// 32-wide K block, which is what tcgen05.mma.kind::mxf8f6f4.block_scale applies
// inside the tensor core: no promotion pass on the CUDA cores, one fp32
// accumulator for the whole K loop.  The 1 x 128 activation / 128 x 128 weight
// recipe of the training path maps onto it by giving every 32-wide sub-block of
// a 128 block the block's exponent; the scale itself is rounded up to a power of
// two when the operand is quantised (at most one bit of fp8 range is lost
// against an fp32 scale, the same trade as the OCP MX formats).
//
// Scale layout in global memory ("SF tiles"): an operand with R rows and K
// columns has ceil(R / 128) x (K / 128) tiles of 512 bytes, tile (rt, kb) at
// byte (rt * K/128 + kb) * 512, and inside it the exponent of row r, 32-wide
// sub-block j at byte (r % 32) * 16 + ((r % 128) / 32) * 4 + j.  That is the
// shared-memory image tcgen05.cp.32x128b.warpx4 copies into tensor memory for
// the MMA: a stage's tiles arrive with a plain bulk copy next to its operand
// tiles, and the MMA-issuing thread moves them to TMEM right before the MMAs
// that read them.
//
// Tile 128 x 256 (one CTA per SM, persistent), K step 128 (one 128-byte swizzle
// row of fp8), 4-stage TMA ring.  Warp 0: TMA producer; warp 1: TMEM owner and
// MMA issuer; warps 2-9: epilogue (a warp = a TMEM lane quarter x 128 columns).
// The 128 x 256 fp32 accumulator and the scale-factor ring share the 512 TMEM
// columns, so there is one accumulator: the epilogue warps load their 128
// columns into registers, release the accumulator at once and do the rounding,
// residual add and stores while the next tile's MMAs already run.  Optional
// fused collectives as in the bf16 GEMM: the all-gather of A (fp8 rows and their
// scale tiles, copied from every rank's staging rows by two copy warps per CTA,
// counted per 128-row chunk) and the reduce-scatter store of the output rows
// into the owners' receive slots.  Every wait is bounded.
//
// Reference: the reference's FP8 support is a per-tensor cast around an fp32
// matmul (include/nn/mixed_precision.hpp:149-196); this is the tensor-core form.
#include "common.cuh"
#include "host_util.h"
#include "lk_api.h"

namespace lk {
namespace {

constexpr int MX_BM = 128, MX_BN = 256, MX_BK = 128;  // BK in elements (= bytes)
constexpr int MX_STAGES = 4;
constexpr int MX_A = MX_BM * MX_BK, MX_B = MX_BN * MX_BK;
constexpr int MX_STAGE = MX_A + MX_B;                 // 48 KB of operands
constexpr int MX_SFA = 512, MX_SFB = 1024;            // scale tiles per stage
constexpr int MX_SF_STAGE = MX_SFA + MX_SFB;
constexpr int MX_EW = 8;                              // epilogue warps
constexpr int MX_THREADS = 64 + 32 * MX_EW;
constexpr int MX_AG_WARPS = 2;
// peer-store staging of the reduce-scatter epilogue: 16 rows x 128 bytes per epilogue warp
constexpr int MX_STG_OFF = MX_STAGES * (MX_STAGE + MX_SF_STAGE) + 256;
constexpr int MX_STG_WARP = 16 * 128;
constexpr int MX_SMEM = MX_STG_OFF + MX_EW * MX_STG_WARP + 1024;
constexpr uint32_t MX_TMEM_COLS = 512;
constexpr uint32_t MX_SF_COL0 = 256;  // scale columns: stage s at 256 + 16 s (A: +0..3, B: +8..15)

struct MxArgs {
  int M, N, K;
  const uint8_t* sfa;  // SF tiles of A: ceil(M/128) x K/128
  const uint8_t* sfb;  // SF tiles of B: 2 ceil(N/256) x K/128
  void* D;
  int64_t ldd;
  const __nv_bfloat16* R;
  int64_t ldr;
  int* status;
  int tiles_m, tiles_n;
  // all-gather of A on first use: rank p's ag_r rows at ag_rows[p] (pitch K)
  // and their SF tiles at ag_sf[p] land in rows [p ag_r, (p+1) ag_r) of a_dst /
  // the matching tiles of sfa_dst; ag_count[c] counts 16-row pieces of chunk c
  const uint8_t* const* ag_rows;
  const uint8_t* const* ag_sf;
  uint8_t* a_dst;
  uint8_t* sfa_dst;
  int ag_r, ag_rank, ag_world;
  int* ag_count;
  // reduce-scatter epilogue: row m -> rptrs[m / rs_rows] at row rs_rank * rs_rows + m % rs_rows
  void* const* rptrs;
  int rs_rows, rs_rank;
};

// tcgen05.cp of 32 rows x 16 bytes (a 512-byte SF tile) into 4 TMEM columns,
// replicated to all four lane quarters.
__device__ __forceinline__ void tc_cp_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// Shared-memory descriptor of a 512-byte SF tile: no swizzle, 16-byte rows,
// 8-row core matrices 128 bytes apart.
__device__ __forceinline__ uint64_t make_desc_sf(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)(128 >> 4) << 16;
  d |= (uint64_t)(128 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  return d;
}

// Instruction descriptor, kind::mxf8f6f4 with UE8M0 scales:
//   [4,6) B scale byte, [7,10) A fmt, [10,13) B fmt, [17,23) N >> 3,
//   [23] scale format (1 = UE8M0), [24,29) M >> 4, [29,31) A scale byte.
__host__ __device__ constexpr uint32_t make_idesc_mxf8(int M, int N, int a_fmt, int b_fmt) {
  return ((uint32_t)a_fmt << 7) | ((uint32_t)b_fmt << 10) | ((uint32_t)(N >> 3) << 17) | (1u << 23) |
         ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void tc_mma_mxf8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %6, 0;\n"
      " tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale.scale_vec::1X [%0], %1, %2, %3, [%4], [%5], p;\n}\n" ::
          "r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(sfa_tmem), "r"(sfb_tmem), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ int mx_ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void mx_fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// bounded wait for a gathered 128-row chunk (8 pieces of 16 rows)
__device__ __forceinline__ bool mx_wait_chunk(const MxArgs& a, int tm, volatile int* abort_flag) {
  const int* cnt = a.ag_count + tm;
  const uint64_t t0 = globaltimer();
  while (mx_ld_acquire(cnt) < 8) {
    if (*abort_flag) return false;
    if (globaltimer() - t0 > LK_WAIT_TIMEOUT_NS) {
      atomicCAS(a.status, 0, LK_ERR_TIMEOUT_PEER);
      *abort_flag = 1;
      return false;
    }
    __nanosleep(100);
  }
  mx_fence_proxy_async_global();
  return true;
}

// Copy warps: 16-row pieces (own rows first, then rank+1, ...) of fp8 rows; the
// first piece of each 128-row chunk also copies the chunk's SF tiles.
__device__ __forceinline__ void mx_ag_copy(const MxArgs& a, int cw, int ncw, int lane) {
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
    if ((r0 & 127) == 0) {
      const uint4* ss = reinterpret_cast<const uint4*>(a.ag_sf[p] + (int64_t)(r0 / 128) * KB * 512);
      uint4* ds = reinterpret_cast<uint4*>(a.sfa_dst + (int64_t)((p * R + r0) / 128) * KB * 512);
      for (int u = lane; u < KB * 32; u += 32) ds[u] = ss[u];
    }
    mx_fence_proxy_async_global();
    __threadfence();
    __syncwarp();
    if (lane == 0) atomicAdd(a.ag_count + (p * R + r0) / 128, 1);
  }
}

__device__ __forceinline__ void mx_tile(int t, int tiles_m, int tiles_n, int& tm, int& tn) {
  constexpr int G = 16;
  const int group = t / (G * tiles_n);
  const int first_m = group * G;
  const int gsz = min(tiles_m - first_m, G);
  const int r = t - group * G * tiles_n;
  tm = first_m + r % gsz;
  tn = r / gsz;
}

template <int AFMT, int BFMT, bool AG, bool REMOTE>
__global__ void __launch_bounds__(MX_THREADS + (AG ? 32 * MX_AG_WARPS : 0), 1)
    gemm_mxf8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const MxArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t sfbase = sbase + MX_STAGES * MX_STAGE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + MX_STAGES * (MX_STAGE + MX_SF_STAGE));
  const uint32_t full0 = smem_u32(bars);
  const uint32_t empty0 = full0 + 8 * MX_STAGES;
  const uint32_t acc_full = empty0 + 8 * MX_STAGES;
  const uint32_t acc_empty = acc_full + 8;
  const uint32_t drain_bar = acc_empty + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * MX_STAGES + 3);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < MX_STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, MX_EW);
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), MX_TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int T = args.tiles_m * args.tiles_n;
  const int nk = args.K / MX_BK;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0, pending = 0, parbits = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < T && ok; t += gridDim.x) {
        int tm, tn;
        mx_tile(t, args.tiles_m, args.tiles_n, tm, tn);
        if constexpr (AG) {
          tm = (tm + args.ag_rank * (args.ag_r / MX_BM)) % args.tiles_m;  // own rows first
          if (!mx_wait_chunk(args, tm, abort_flag)) {
            ok = false;
            break;
          }
        }
        const uint8_t* sfa_t = args.sfa + (int64_t)tm * nk * 512;
        const uint8_t* sfb_t0 = args.sfb + (int64_t)(2 * tn) * nk * 512;
        const uint8_t* sfb_t1 = sfb_t0 + (int64_t)nk * 512;
        for (int kb = 0; kb < nk; ++kb) {
          if (!bounded_wait(empty0 + 8 * s, ph ^ 1, args.status, LK_ERR_TIMEOUT_EMPTY, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t fb = full0 + 8 * s;
          const uint32_t sa = sbase + s * MX_STAGE;
          const uint32_t sf = sfbase + s * MX_SF_STAGE;
          mbar_expect_tx(fb, MX_STAGE + MX_SF_STAGE);
          tma_load_2d(sa, &tmA, fb, kb * MX_BK, tm * MX_BM);
          tma_load_2d(sa + MX_A, &tmB, fb, kb * MX_BK, tn * MX_BN);
          bulk_load(sf, sfa_t + kb * 512, 512, fb);
          bulk_load(sf + MX_SFA, sfb_t0 + kb * 512, 512, fb);
          bulk_load(sf + MX_SFA + 512, sfb_t1 + kb * 512, 512, fb);
          pending |= 1u << s;
          parbits = (parbits & ~(1u << s)) | (ph << s);
          if (++s == MX_STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      if (!ok)
        for (int i = 0; i < MX_STAGES; ++i)
          if (pending & (1u << i))
            bounded_wait(full0 + 8 * i, (parbits >> i) & 1, args.status, LK_ERR_TIMEOUT_DRAIN, nullptr);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_mxf8(MX_BM, MX_BN, AFMT, BFMT);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      int local = 0;
      for (int t = blockIdx.x; t < T && ok; t += gridDim.x, ++local) {
        // the epilogue has moved the previous tile's accumulator into registers
        if (!bounded_wait(acc_empty, (local & 1) ^ 1, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kb = 0; kb < nk; ++kb) {
          if (!bounded_wait(full0 + 8 * s, ph, args.status, LK_ERR_TIMEOUT_FULL, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = sbase + s * MX_STAGE;
          const uint32_t sb = sa + MX_A;
          const uint32_t sf = sfbase + s * MX_SF_STAGE;
          const uint32_t tsfa = tmem + MX_SF_COL0 + 16 * s;
          const uint32_t tsfb = tsfa + 8;
          // scale tiles to TMEM; tcgen05.cp and tcgen05.mma of one thread run in order
          tc_cp_sf(tsfa, make_desc_sf(sf));
          tc_cp_sf(tsfb, make_desc_sf(sf + MX_SFA));
          tc_cp_sf(tsfb + 4, make_desc_sf(sf + MX_SFA + 512));
#pragma unroll
          for (int kk = 0; kk < MX_BK / 32; ++kk)
            tc_mma_mxf8(tmem, make_desc_sw128(sa + kk * 32, 16, 1024), make_desc_sw128(sb + kk * 32, 16, 1024),
                        idesc | ((uint32_t)kk << 29) | ((uint32_t)kk << 4), tsfa, tsfb, (kb | kk) != 0 ? 1u : 0u);
          tc_commit(empty0 + 8 * s);
          if (++s == MX_STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
        if (ok) tc_commit(acc_full);
      }
      tc_commit(drain_bar);
      bounded_wait(drain_bar, 0, args.status, LK_ERR_TIMEOUT_DRAIN, nullptr);
    }
  } else if (AG && warp >= 2 + MX_EW) {
    // ---------------------------------------------------------- copy warps
    mx_ag_copy(args, (warp - 2 - MX_EW) * gridDim.x + blockIdx.x, MX_AG_WARPS * gridDim.x, lane);
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;           // TMEM lane quarter this warp may read
    const int h = (warp - 2) >> 2;    // column half of the tile
    const int row_in_tile = q * 32 + lane;
    int local = 0;
    for (int t = blockIdx.x; t < T; t += gridDim.x, ++local) {
      int tm, tn;
      mx_tile(t, args.tiles_m, args.tiles_n, tm, tn);
      if constexpr (AG) tm = (tm + args.ag_rank * (args.ag_r / MX_BM)) % args.tiles_m;
      const bool ok = bounded_wait(acc_full, local & 1, args.status, LK_ERR_TIMEOUT_ACCUM, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      uint32_t r[4][32];
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + h * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(taddr + 32 * c, r[c]);
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);  // the MMAs of the next tile may start
      const int row = tm * MX_BM + row_in_tile;
      // bf16 values of this lane's row, 16 chunks of 8 columns (+ residual)
      uint4 pk[16];
#pragma unroll
      for (int v = 0; v < 16; ++v) {
        const int col = tn * MX_BN + h * 128 + v * 8;
        float f[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(r[v >> 2][(v & 3) * 8 + e]);
        if (args.R && row < args.M && col < args.N) {
          const uint4 rv = *reinterpret_cast<const uint4*>(args.R + (int64_t)row * args.ldr + col);
          const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 x = unpack_bf16x2(rw[e]);
            f[2 * e] += x.x;
            f[2 * e + 1] += x.y;
          }
        }
        pk[v] = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                           pack_bf16x2(f[6], f[7]));
      }
      if constexpr (REMOTE) {
        // Rows go to their owners over NVLink.  Stored thread-per-row, each
        // instruction would send 32 separate 16-byte pieces; instead 16 rows x
        // 128 bytes at a time pass through this warp's shared-memory slot
        // (16-byte chunks XOR-swizzled by row) and leave as whole 128-byte row
        // segments, 8 lanes per row.
        uint8_t* stg = smem + MX_STG_OFF + (warp - 2) * MX_STG_WARP;
#pragma unroll
        for (int rh = 0; rh < 2; ++rh) {
#pragma unroll
          for (int ch = 0; ch < 2; ++ch) {
            if ((lane >> 4) == rh) {
              const int rl = lane & 15;
#pragma unroll
              for (int c = 0; c < 8; ++c)
                *reinterpret_cast<uint4*>(stg + rl * 128 + ((c ^ (rl & 7)) << 4)) = pk[ch * 8 + c];
            }
            __syncwarp();
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int rl = k * 4 + (lane >> 3), j = lane & 7;
              const uint4 val = *reinterpret_cast<const uint4*>(stg + rl * 128 + ((j ^ (rl & 7)) << 4));
              const int grow = tm * MX_BM + q * 32 + rh * 16 + rl;
              const int col = tn * MX_BN + h * 128 + ch * 64 + j * 8;
              if (grow < args.M && col < args.N) {
                const int owner = grow / args.rs_rows;
                __nv_bfloat16* drow = reinterpret_cast<__nv_bfloat16*>(args.rptrs[owner]) +
                                      (int64_t)(args.rs_rank * args.rs_rows + grow - owner * args.rs_rows) * args.ldd;
                *reinterpret_cast<uint4*>(drow + col) = val;
              }
            }
            __syncwarp();
          }
        }
      } else if (row < args.M) {
        __nv_bfloat16* drow = reinterpret_cast<__nv_bfloat16*>(args.D) + (int64_t)row * args.ldd;
#pragma unroll
        for (int v = 0; v < 16; ++v) {
          const int col = tn * MX_BN + h * 128 + v * 8;
          if (col >= args.N) break;
          *reinterpret_cast<uint4*>(drow + col) = pk[v];
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, MX_TMEM_COLS);
  }
}

// ------------------------------------------------------------ quantisation
// Exponent e (scale 2^e) of a block whose largest magnitude is amax, the
// smallest with amax / 2^e <= the format's largest finite value
// (e4m3: 1.75 * 2^8, e5m2: 1.75 * 2^15); clamped to the UE8M0 range.
__device__ __forceinline__ int mx_exponent(float amax, int fmt) {
  const uint32_t u = __float_as_uint(amax);
  const int E = (int)((u >> 23) & 0xFF) - 127;
  const uint32_t mant = u & 0x7FFFFF;
  int e = E - (fmt == 0 ? 8 : 15) + (mant > 0x600000u ? 1 : 0);
  return max(-127, min(e, 127));
}

// 2^-e for e in [-127, 126], exact
__device__ __forceinline__ float mx_inv_scale(int e) { return __uint_as_float((uint32_t)(127 - e) << 23); }

__device__ __forceinline__ uint8_t mx_to_f8(float v, int fmt) {
  __nv_fp8_storage_t r = fmt == 0 ? __nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3)
                                  : __nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E5M2);
  return (uint8_t)r;
}

__device__ __forceinline__ int64_t mx_sf_offset(int row, int kb, int nkb) {
  return ((int64_t)(row >> 7) * nkb + kb) * 512 + (row & 31) * 16 + ((row & 127) >> 5) * 4;
}

// Activations / gradients, 1 x 128 blocks: a half-warp per (row, K block),
// 8 elements (16 bytes) per lane, grid-stride.  Rows [M, rows_pad) get exponent
// 0 (byte 127) in the SF tiles and no data.
__global__ void __launch_bounds__(256) quant_mx_rows_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int M,
                                                            int rows_pad, int K, int fmt, uint8_t* __restrict__ q,
                                                            int64_t ldq, uint8_t* __restrict__ sf) {
  const int lane = threadIdx.x & 31, sub = lane & 15;
  const uint32_t hmask = lane < 16 ? 0x0000FFFFu : 0xFFFF0000u;
  const int nkb = K / 128;
  const int64_t units = (int64_t)rows_pad * nkb;
  const int64_t stride = ((int64_t)gridDim.x * blockDim.x) >> 4;
  for (int64_t u = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 4; u < units; u += stride) {
    const int row = (int)(u / nkb), kb = (int)(u % nkb);
    if (row >= M) {
      if (sub == 0) *reinterpret_cast<uint32_t*>(sf + mx_sf_offset(row, kb, nkb)) = 0x7F7F7F7Fu;
      continue;
    }
    const uint4 v = *reinterpret_cast<const uint4*>(x + (int64_t)row * ldx + kb * 128 + sub * 8);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    float f[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 t = unpack_bf16x2(w[e]);
      f[2 * e] = t.x;
      f[2 * e + 1] = t.y;
    }
    float amax = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(f[e]));
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(hmask, amax, o));
    const int ex = mx_exponent(amax, fmt);
    const float inv = mx_inv_scale(ex);
    uint32_t pk[2];
#pragma unroll
    for (int h = 0; h < 2; ++h)
      pk[h] = (uint32_t)mx_to_f8(f[4 * h] * inv, fmt) | ((uint32_t)mx_to_f8(f[4 * h + 1] * inv, fmt) << 8) |
              ((uint32_t)mx_to_f8(f[4 * h + 2] * inv, fmt) << 16) | ((uint32_t)mx_to_f8(f[4 * h + 3] * inv, fmt) << 24);
    *reinterpret_cast<uint2*>(q + (int64_t)row * ldq + kb * 128 + sub * 8) = make_uint2(pk[0], pk[1]);
    if (sub == 0) *reinterpret_cast<uint32_t*>(sf + mx_sf_offset(row, kb, nkb)) = (uint32_t)(ex + 127) * 0x01010101u;
  }
}

// Weights, 128 x 128 blocks of e4m3: one block per tile.  Writes W8 [N, K], its
// SF tiles, the fp32 scales 2^e [ceil(N/128), K/128] and, when qt is given,
// W8^T [K, N] with its SF tiles (the dgrad operand; same block exponents).
__global__ void __launch_bounds__(256) quant_mx_128x128_kernel(const __nv_bfloat16* __restrict__ w, int64_t ldw,
                                                               int N, int K, uint8_t* __restrict__ q,
                                                               uint8_t* __restrict__ sf, float* __restrict__ scale,
                                                               uint8_t* __restrict__ qt, uint8_t* __restrict__ sft) {
  __shared__ float red[8];
  __shared__ int e_sh;
  __shared__ uint8_t tile[128][129];
  const int nb = blockIdx.y, kb = blockIdx.x;
  const int nkb = K / 128, nnb = (N + 127) / 128;
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
    const int e = mx_exponent(m, 0);
    e_sh = e;
    scale[(int64_t)nb * nkb + kb] = __uint_as_float((uint32_t)(e + 127) << 23);
  }
  __syncthreads();
  const int e = e_sh;
  const float inv = mx_inv_scale(e);
  const uint32_t word = (uint32_t)(e + 127) * 0x01010101u;
  if (threadIdx.x < 128) {
    reinterpret_cast<uint32_t*>(sf + ((int64_t)nb * nkb + kb) * 512)[threadIdx.x] = word;
    if (sft) reinterpret_cast<uint32_t*>(sft + ((int64_t)kb * nnb + nb) * 512)[threadIdx.x] = word;
  }
  for (int i = threadIdx.x; i < 128 * 128; i += 256) {
    const int r = i / 128, c = i % 128;
    const int n = nb * 128 + r;
    uint8_t v = 0;
    if (n < N) {
      v = mx_to_f8(__bfloat162float(w[(int64_t)n * ldw + kb * 128 + c]) * inv, 0);
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

// x = q * 2^e (SF tiles, one exponent per row and 128-wide K block: byte 0 of
// the block's four) -> bf16; one thread per 8 elements.
__global__ void __launch_bounds__(256) dequant_mx_rows_kernel(const uint8_t* __restrict__ q, int M, int K, int fmt,
                                                              const uint8_t* __restrict__ sf,
                                                              __nv_bfloat16* __restrict__ x, int64_t ldx) {
  const int64_t n8 = (int64_t)M * K / 8;
  const int nkb = K / 128;
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < n8; u += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = u * 8;
    const int row = (int)(e / K), col = (int)(e % K);
    const int ex = (int)sf[mx_sf_offset(row, col / 128, nkb) + (col & 127) / 32] - 127;
    const float sc = __uint_as_float((uint32_t)(ex + 127) << 23);
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

extern "C" int lk_dequant_mx_rows(const void* q, int M, int K, int fmt, const void* sf, void* x, int64_t ldx,
                                  cudaStream_t s) {
  LK_REQUIRE(K % 128 == 0 && ldx % 8 == 0, "dequant_mx_rows: K % 128, ldx % 8");
  const int64_t n8 = (int64_t)M * K / 8;
  if (n8 == 0) return 0;
  const int grid = (int)std::min<int64_t>((n8 + 255) / 256, 8 * num_sms());
  dequant_mx_rows_kernel<<<grid, 256, 0, s>>>((const uint8_t*)q, M, K, fmt, (const uint8_t*)sf,
                                              (__nv_bfloat16*)x, ldx);
  return check_launch("dequant_mx_rows");
}

extern "C" int lk_gemm_mxf8(const LkGemmMxf8Desc* g, cudaStream_t stream) {
  LK_REQUIRE(g->K % 128 == 0 && g->K > 0, "gemm_mxf8: K must be a positive multiple of 128");
  LK_REQUIRE(g->N % 8 == 0 && g->a_ld % 16 == 0 && g->b_ld % 16 == 0 && g->ldd % 8 == 0,
             "gemm_mxf8: N % 8, operand pitch % 16 bytes, output pitch % 8");
  LK_REQUIRE((g->a_fmt == 0 || g->a_fmt == 1) && (g->b_fmt == 0 || g->b_fmt == 1),
             "gemm_mxf8: formats e4m3 (0) or e5m2 (1)");
  LK_REQUIRE(g->sfa && g->sfb, "gemm_mxf8: scale tiles required");
  LK_REQUIRE(((uintptr_t)g->sfa & 15) == 0 && ((uintptr_t)g->sfb & 15) == 0, "gemm_mxf8: SF tiles 16-byte aligned");
  if (g->M == 0 || g->N == 0) return 0;
  MxArgs a{};
  a.M = g->M;
  a.N = g->N;
  a.K = g->K;
  a.sfa = reinterpret_cast<const uint8_t*>(g->sfa);
  a.sfb = reinterpret_cast<const uint8_t*>(g->sfb);
  a.D = g->d;
  a.ldd = g->ldd;
  a.R = reinterpret_cast<const __nv_bfloat16*>(g->r);
  a.ldr = g->ldr;
  a.status = g->status;
  a.tiles_m = cdiv(g->M, MX_BM);
  a.tiles_n = cdiv(g->N, MX_BN);
  CUtensorMap ta, tb;
  const CUtensorMapDataType u8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  if (!make_tmap_2d(&ta, g->a, u8, 1, g->M, g->K, g->a_ld, MX_BM, MX_BK)) return -1;
  if (!make_tmap_2d(&tb, g->b, u8, 1, g->N, g->K, g->b_ld, MX_BN, MX_BK)) return -1;
  a.ag_rows = reinterpret_cast<const uint8_t* const*>(g->ag_rows);
  a.ag_sf = reinterpret_cast<const uint8_t* const*>(g->ag_sf);
  a.a_dst = reinterpret_cast<uint8_t*>(const_cast<void*>(g->a));
  a.sfa_dst = reinterpret_cast<uint8_t*>(const_cast<void*>(g->sfa));
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
    LK_REQUIRE(g->ag_count && g->ag_sf && g->ag_rows_per_rank % 128 == 0 &&
                   (int64_t)g->ag_rows_per_rank * g->world == g->M && g->a_ld == g->K,
               "gemm_mxf8 all-gather: M = world x rows (rows % 128 == 0), dense A");
    if (cudaMemsetAsync(g->ag_count, 0, sizeof(int) * a.tiles_m, stream) != cudaSuccess)
      return fail("gemm_mxf8: memset failed");
  }
  if (remote) LK_REQUIRE(g->rs_rows > 0 && g->M % g->rs_rows == 0, "gemm_mxf8 reduce-scatter: M = world x rs_rows");
  LK_REQUIRE(!(ag && remote), "gemm_mxf8: all-gather and reduce-scatter modes are exclusive");
  void* kern = nullptr;
#define LK_MX_PICK(FA, FB, AGV, RV) \
  if (g->a_fmt == FA && g->b_fmt == FB && ag == AGV && remote == RV) kern = (void*)gemm_mxf8_kernel<FA, FB, AGV, RV>;
  LK_MX_PICK(0, 0, false, false) LK_MX_PICK(1, 0, false, false) LK_MX_PICK(0, 1, false, false)
  LK_MX_PICK(1, 1, false, false) LK_MX_PICK(0, 0, true, false) LK_MX_PICK(0, 0, false, true)
  LK_MX_PICK(1, 0, true, false) LK_MX_PICK(1, 0, false, true)
#undef LK_MX_PICK
  LK_REQUIRE(kern != nullptr, "gemm_mxf8: fused collectives take an e4m3 B operand");
  static uint64_t attr_set[12] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  const int variant = (g->a_fmt * 2 + g->b_fmt) + (ag ? 4 : 0) + (remote ? 8 : 0);
  if (!(attr_set[variant] & (1ull << dev))) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, MX_SMEM);
    attr_set[variant] |= 1ull << dev;
  }
  void* params[] = {&ta, &tb, &a};
  if (ag) {
    // CTAs wait on rows copied by other CTAs: all of them must be resident
    cudaError_t e = cudaLaunchCooperativeKernel(kern, dim3(grid), dim3(MX_THREADS + 32 * MX_AG_WARPS), params,
                                                MX_SMEM, stream);
    if (e != cudaSuccess) {
      last_error() = std::string("gemm_mxf8 cooperative launch: ") + cudaGetErrorString(e);
      return -1;
    }
  } else {
    cudaError_t e = cudaLaunchKernel(kern, dim3(grid), dim3(MX_THREADS), params, MX_SMEM, stream);
    if (e != cudaSuccess) {
      last_error() = std::string("gemm_mxf8 launch: ") + cudaGetErrorString(e);
      return -1;
    }
  }
  return check_launch("gemm_mxf8");
}

extern "C" int lk_quant_mx_rows(const void* x, int64_t ldx, int M, int rows_pad, int K, int fmt, void* q,
                                int64_t ldq, void* sf, cudaStream_t s) {
  LK_REQUIRE(K % 128 == 0 && ldx % 8 == 0 && ldq % 8 == 0, "quant_mx_rows: K % 128, aligned pitches");
  LK_REQUIRE(rows_pad >= M && rows_pad % 128 == 0, "quant_mx_rows: rows_pad >= M, multiple of 128");
  LK_REQUIRE(fmt == 0 || fmt == 1, "quant_mx_rows: e4m3 (0) or e5m2 (1)");
  LK_REQUIRE(ldq % 8 == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)q & 7) == 0,
             "quant_mx_rows: 16-byte aligned x rows, 8-byte aligned q rows");
  const int64_t units = (int64_t)rows_pad * (K / 128);
  if (units == 0) return 0;
  const int grid = (int)std::min<int64_t>((units + 15) / 16, (int64_t)num_sms() * 16);
  quant_mx_rows_kernel<<<grid, 256, 0, s>>>((const __nv_bfloat16*)x, ldx, M, rows_pad, K, fmt, (uint8_t*)q, ldq,
                                           (uint8_t*)sf);
  return check_launch("quant_mx_rows");
}

extern "C" int lk_quant_mx_128x128(const void* w, int64_t ldw, int N, int K, void* q, void* sf, float* scale,
                                   void* qt, void* sft, cudaStream_t s) {
  LK_REQUIRE(K % 128 == 0 && N % 16 == 0, "quant_mx_128x128: K % 128, N % 16");
  LK_REQUIRE(!qt || N % 128 == 0, "quant_mx_128x128: the transposed copy needs N % 128 == 0");
  dim3 grid(K / 128, (N + 127) / 128);
  quant_mx_128x128_kernel<<<grid, 256, 0, s>>>((const __nv_bfloat16*)w, ldw, N, K, (uint8_t*)q, (uint8_t*)sf, scale,
                                               (uint8_t*)qt, (uint8_t*)sft);
  return check_launch("quant_mx_128x128");
}
