// K1: bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
//   D[M, N] = alpha * A[M, K] . B[N, K]^T   (+ fused epilogue)
//
// A and B are each either K-major (row-major with K contiguous) or MN-major
// (the transpose view of a row-major [K, M] / [K, N] tensor), which covers the
// three GEMMs of a linear layer without any transpose copies:
//   forward  Y  = X  W^T      A K-major,  B K-major
//   dgrad    dX = dY W        A K-major,  B MN-major (W^T view)
//   wgrad    dW = dY^T X      A MN-major, B MN-major
//
// Design (one CTA per SM, persistent over output tiles):
//   warp 0      one thread issues TMA tile loads (128B swizzle, no multicast)
//               into a STAGES-deep shared-memory ring guarded by mbarriers;
//   warp 1      one thread issues tcgen05.mma (M=128, N=BN, K=16) into a
//               double-buffered fp32 TMEM accumulator and tcgen05.commit's the
//               stage back to the producer;
//   warps 2..5  the epilogue: tcgen05.ld 32 lanes x 32 columns per warp, apply
//               the fused epilogue, store to global; overlaps the next tile's
//               MMAs thanks to the second accumulator buffer.
// Every wait is bounded (see common.cuh): on timeout the CTA records a status
// code, drains its in-flight TMA copies and MMAs, frees TMEM and returns.
//
// Replaces the reference's scalar/cuBLAS GEMMs: GemmEngine::matmul
// (include/core/gemm_engine.hpp:30-55), gemm_tiled_kernel
// (include/hw/cuda_kernels.hpp:18-50) and the matmul loops of
// src/nn/transformer_blocks.cpp (QKV :22-38, FFN :264-302, LM head :659-667).
#pragma once
#include "common.cuh"
#include "host_util.h"
#include "lk_api.h"

namespace lk {

enum GemmEpi : int {
  EPI_BF16 = 0,        // D(bf16) = alpha*acc
  EPI_F32 = 1,         // D(f32)  = alpha*acc
  EPI_F32_ACC = 2,     // D(f32) += alpha*acc          (gradient accumulation)
  EPI_BF16_RESID = 3,  // D(bf16) = alpha*acc + R(bf16) (residual add; D may alias R)
  EPI_SWIGLU = 4,      // D(bf16) = acc (gate|up), H(bf16) = silu(gate) * up
  EPI_REMOTE = 5,      // K18: bf16 tile stored into the owner rank's receive slot (peer memory)
  EPI_SWIGLU_BWD = 6,  // acc = dh; D(bf16 [M, 2N] gate|up grads) from R (gate|up), dh not stored
  EPI_BF16_ROPE = 7,   // D(bf16) = alpha*acc, columns < rope_cols rotated (RoPE) first
};

struct GemmArgs {
  int M, N, K;
  void* D;
  int64_t ldd;
  const __nv_bfloat16* R;
  int64_t ldr;
  __nv_bfloat16* H;
  int64_t ldh;
  float alpha;
  int* status;
  int tiles_m, tiles_n;
  int K2;  // > 0: a second contraction segment (A2 . B2^T) accumulated into the same tile
  int m_rot;  // M-tile rotation: rank r starts at M-tile m_rot (staggers peers' traffic)
  // K18 remote-store epilogue: row m belongs to owner m / rs_rows and lands in
  // rptrs[owner] at row (rs_rank * rs_rows + m % rs_rows), pitch ldd
  void* const* rptrs;
  const CUtensorMap* rmaps;  // optional: per-owner tensor maps of the receive buffers (TMA stores)
  int rs_rows, rs_rank;
  // K16 all-gather of A on first use: rank p's rows [0, ag_rows) live at
  // ag_src[p] (pitch ag_ld_src bytes; p == ag_rank is this GPU's own staging
  // rows) and are copied into rows [p*ag_rows, (p+1)*ag_rows) of the local A
  // buffer ag_dst (pitch ag_ld_dst bytes) by the copy warps; ag_count[c]
  // counts copied 16-row pieces of the 128-row chunk c (8 = ready).
  const uint8_t* const* ag_src;
  int64_t ag_ld_src, ag_ld_dst;
  uint8_t* ag_dst;
  int ag_rows, ag_rank, ag_world, ag_row_bytes;
  int* ag_count;
  // K17 gather of a flat parameter group on first use (ZeRO-3): rank p owns
  // group elements [p*gb_chunk, (p+1)*gb_chunk) at gb_src[p] (bf16); the copy
  // warps assemble the whole group (gb_len elements) at gb_dst, B being the
  // [N, K] tensor at element gb_boff of it.  gb_count[tn] counts the copied
  // GB_PIECE-element pieces that overlap N-tile tn's part of B.
  const uint8_t* const* gb_src;
  int64_t gb_chunk, gb_len, gb_boff;
  uint8_t* gb_dst;
  int* gb_count;
  // EPI_BF16_ROPE: (cos, sin) table [max_pos, rope_dh / 2], rotated columns, position = row % seq + off
  const float2* rope_table;
  int rope_cols, rope_dh, rope_seq, rope_off;
};

constexpr int64_t GB_PIECE = 8192;  // elements per K17 copy piece (16 KB)

constexpr int AG_SUB = 16;  // rows per copy piece

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;
constexpr int GEMM_THREADS = 192;

// CG = 2: a CTA pair (cluster of 2) computes a 256 x BN tile with
// tcgen05.mma.cta_group::2; each CTA loads its own 128 rows of A and its half
// of B's BN rows (plain TMA, no multicast), so per CTA the operand bytes per
// FLOP drop by a third against the single-CTA 128 x BN tile.
template <int BN, int CG = 1>
struct GemmCfg {
  static constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;
  static constexpr int B_BYTES = (BN / CG) * GEMM_BK * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int STAGES = CG == 1 ? ((BN == 256) ? 4 : 6) : (196608 / STAGE > 8 ? 8 : 196608 / STAGE);
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM = STAGES * STAGE + BAR_BYTES + 1024;
  static constexpr int TMEM_COLS = 2 * BN;
};

// Grouped tile order: GROUP consecutive M-tiles share each sweep over N so the
// B panel and the A rows they use stay resident in L2.
__device__ __forceinline__ void gemm_tile_coords(int t, int tiles_m, int tiles_n, int& tm,
                                                 int& tn) {
  constexpr int G = 16;
  const int group = t / (G * tiles_n);
  const int first_m = group * G;
  const int gsz = min(tiles_m - first_m, G);
  const int r = t - group * G * tiles_n;
  tm = first_m + r % gsz;
  tn = r / gsz;
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// K16 copy warps (AG_WARPS per CTA): pull the gathered rows of A into the
// local buffer, one 16-row piece at a time.  Pieces are numbered own rows
// first, then rank+1, rank+2, ... (the M-tile order of the GEMM), and dealt
// round-robin over every copy warp of the grid so the first pieces land on
// all SMs at once.  Each lane keeps 16 x 16-byte loads in flight per row.
constexpr int AG_WARPS = 2;

__device__ __forceinline__ void ag_copy_warp(const GemmArgs& a, int cw, int ncw, int lane) {
  const int R = a.ag_rows, W = a.ag_world, me = a.ag_rank;
  const int per_rank = R / AG_SUB;
  const int total = per_rank * W;
  const int upr = a.ag_row_bytes / 16;  // 16-byte units per row
  for (int s = cw; s < total; s += ncw) {
    const int p = (me + s / per_rank) % W;
    const int r0 = (s % per_rank) * AG_SUB;
    const uint8_t* src = a.ag_src[p] + (int64_t)r0 * a.ag_ld_src;
    uint8_t* dst = a.ag_dst + (int64_t)(p * R + r0) * a.ag_ld_dst;
#pragma unroll 1
    for (int r = 0; r < AG_SUB; ++r) {
      const uint4* sr = reinterpret_cast<const uint4*>(src + (int64_t)r * a.ag_ld_src);
      uint4* dr = reinterpret_cast<uint4*>(dst + (int64_t)r * a.ag_ld_dst);
#pragma unroll 1
      for (int c0 = lane; c0 < upr; c0 += 32 * 16) {
        uint4 v[16];
#pragma unroll
        for (int k = 0; k < 16; ++k)
          if (c0 + 32 * k < upr) v[k] = sr[c0 + 32 * k];
#pragma unroll
        for (int k = 0; k < 16; ++k)
          if (c0 + 32 * k < upr) dr[c0 + 32 * k] = v[k];
      }
    }
    fence_proxy_async_global();  // the rows are read next by TMA (async proxy)
    __threadfence();
    __syncwarp();
    if (lane == 0) atomicAdd(a.ag_count + (p * R + r0) / 128, 1);
  }
}

// Producer side of K16/K17: wait (bounded) until *cnt reaches target, then
// order the async-proxy (TMA) reads after the copies it counts.
__device__ __forceinline__ bool wait_count(const GemmArgs& a, const int* cnt, int target,
                                           volatile int* abort_flag) {
  if (ld_acquire_gpu(cnt) >= target) {
    fence_proxy_async_global();
    return true;
  }
  const uint64_t t0 = globaltimer();
  while (true) {
    for (int i = 0; i < 64; ++i) {
      if (ld_acquire_gpu(cnt) >= target) {
        fence_proxy_async_global();
        return true;
      }
      __nanosleep(100);
    }
    if (*abort_flag) return false;
    if (globaltimer() - t0 > LK_WAIT_TIMEOUT_NS) {
      atomicCAS(a.status, 0, LK_ERR_TIMEOUT_PEER);
      *abort_flag = 1;
      return false;
    }
  }
}

// K17: the part of the group that N-tile tn of B reads: [lo, hi) elements.
// K-major B reads rows [tn*BN, (tn+1)*BN); MN-major B reads every row.
template <int BN, bool B_MN>
__device__ __forceinline__ void gb_tile_range(const GemmArgs& a, int tn, int64_t& lo, int64_t& hi) {
  const int64_t nk = (int64_t)a.N * a.K;
  if (B_MN) {
    lo = a.gb_boff;
    hi = a.gb_boff + nk;
  } else {
    lo = a.gb_boff + (int64_t)tn * BN * a.K;
    hi = a.gb_boff + min((int64_t)(tn + 1) * BN * a.K, nk);
  }
}

// K17 copy warps: pieces of the group in order - B's pieces first (each rank
// starting at a different one so the owners' links share the load), then the
// rest.  A piece may straddle two owners' chunks.
template <int BN, bool B_MN>
__device__ __forceinline__ void gb_copy_warp(const GemmArgs& a, int cw, int ncw, int lane, int rank,
                                             int world) {
  const int64_t npieces = (a.gb_len + GB_PIECE - 1) / GB_PIECE;
  const int64_t pb0 = a.gb_boff / GB_PIECE;
  const int64_t pb1 = (a.gb_boff + (int64_t)a.N * a.K - 1) / GB_PIECE;
  const int64_t nb = pb1 - pb0 + 1;
  const int64_t rot = nb * rank / world;
  for (int64_t s = cw; s < npieces; s += ncw) {
    int64_t piece;
    if (s < nb) {
      piece = pb0 + (s + rot) % nb;
    } else {
      const int64_t k = s - nb;
      piece = k < pb0 ? k : k + nb;
    }
    const int64_t a0 = piece * GB_PIECE;
    const int64_t a1 = min(a0 + GB_PIECE, a.gb_len);
    int64_t e = a0;
    while (e < a1) {
      const int64_t p = e / a.gb_chunk;
      const int64_t seg_end = min(a1, (p + 1) * a.gb_chunk);
      const uint4* src = reinterpret_cast<const uint4*>(a.gb_src[p] + (e - p * a.gb_chunk) * 2);
      uint4* dst = reinterpret_cast<uint4*>(a.gb_dst + e * 2);
      const int units = (int)((seg_end - e) / 8);
#pragma unroll 1
      for (int c0 = lane; c0 < units; c0 += 32 * 8) {
        uint4 v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (c0 + 32 * k < units) v[k] = src[c0 + 32 * k];
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (c0 + 32 * k < units) dst[c0 + 32 * k] = v[k];
      }
      e = seg_end;
    }
    fence_proxy_async_global();
    __threadfence();
    __syncwarp();
    if (lane == 0) {
      // count this piece for every N-tile whose part of B it overlaps
      const int tiles_n = (a.N + BN - 1) / BN;
      for (int tn = 0; tn < tiles_n; ++tn) {
        int64_t lo, hi;
        gb_tile_range<BN, B_MN>(a, tn, lo, hi);
        if (a0 < hi && a1 > lo) atomicAdd(a.gb_count + tn, 1);
      }
    }
  }
}

template <int BN, bool B_MN>
__device__ __forceinline__ int gb_expected(const GemmArgs& a, int tn) {
  int64_t lo, hi;
  gb_tile_range<BN, B_MN>(a, tn, lo, hi);
  return (int)((hi - 1) / GB_PIECE - lo / GB_PIECE + 1);
}

template <int BN, bool A_MN, bool B_MN, int EPI, int AG = 0, int CG = 1>
__global__ void __launch_bounds__(AG ? GEMM_THREADS + 32 * AG_WARPS : GEMM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2,
                   const GemmArgs args) {
  using C = GemmCfg<BN, CG>;
  static_assert(CG == 1 || (AG == 0 && EPI != EPI_REMOTE), "CTA pairs: plain epilogues only");
  constexpr int BM_T = GEMM_BM * CG;  // rows of one output tile
  constexpr int BNH = BN / CG;         // rows of B this CTA loads
  const uint32_t crank = CG == 2 ? cluster_ctarank() : 0u;  // 0: leader (issues the MMAs)
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  const uint32_t sbase = smem_u32(smem);

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE);
  const uint32_t full0 = smem_u32(bars);
  const uint32_t empty0 = full0 + 8 * C::STAGES;
  const uint32_t tfull0 = empty0 + 8 * C::STAGES;
  const uint32_t tempty0 = tfull0 + 16;
  const uint32_t drain_bar = tempty0 + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * C::STAGES + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull0 + 8 * b, 1);
      mbar_init(tempty0 + 8 * b, 4 * CG);  // every epilogue warp of the pair arrives on the leader's
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (args.K2 > 0) {
      tma_prefetch_desc(&tmA2);
      tma_prefetch_desc(&tmB2);
    }
  }
  if (warp == 1) {
    if constexpr (CG == 2)
      tmem_alloc_pair(smem_u32(tmem_slot), C::TMEM_COLS);
    else
      tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
  }
  tc_fence_before();
  if constexpr (CG == 2)
    cluster_sync();  // the peer's barriers are initialised before any remote arrive / complete_tx
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int T = args.tiles_m * args.tiles_n;
  // persistent tile loop: a pair walks the tiles as one unit
  const int t_first = CG == 2 ? (int)(blockIdx.x / 2) : (int)blockIdx.x;
  const int t_step = CG == 2 ? (int)(gridDim.x / 2) : (int)gridDim.x;
  const int nk1 = (args.K + GEMM_BK - 1) / GEMM_BK;
  const int nk = nk1 + (args.K2 > 0 ? (args.K2 + GEMM_BK - 1) / GEMM_BK : 0);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0, pending = 0, parbits = 0;
      bool ok = true;
      for (int t = t_first; t < T && ok; t += t_step) {
        int tm, tn;
        gemm_tile_coords(t, args.tiles_m, args.tiles_n, tm, tn);
        tm = (tm + args.m_rot) % args.tiles_m;
        const int arow = tm * BM_T + (int)crank * GEMM_BM;  // this CTA's rows of A
        const int brow = tn * BN + (int)crank * BNH;        // this CTA's rows of B
        if constexpr (AG == 1) {
          if (!wait_count(args, args.ag_count + tm, 128 / AG_SUB, abort_flag)) {
            ok = false;
            break;
          }
        } else if constexpr (AG == 2) {
          if (!wait_count(args, args.gb_count + tn, gb_expected<BN, B_MN>(args, tn), abort_flag)) {
            ok = false;
            break;
          }
        }
        for (int kb = 0; kb < nk; ++kb) {
          if (!bounded_wait(empty0 + 8 * s, ph ^ 1, args.status, LK_ERR_TIMEOUT_EMPTY,
                            abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t fb = full0 + 8 * s;
          const uint32_t sa = sbase + s * C::STAGE;
          const uint32_t sb = sa + C::A_BYTES;
          // k-blocks [0, nk1) come from (A, B), the rest from the second segment (A2, B2)
          const bool seg2 = kb >= nk1;
          const CUtensorMap* ma = seg2 ? &tmA2 : &tmA;
          const CUtensorMap* mb = seg2 ? &tmB2 : &tmB;
          const int kc = (seg2 ? kb - nk1 : kb) * GEMM_BK;
          if constexpr (CG == 1) {
            mbar_expect_tx(fb, C::STAGE);
            if (!A_MN) {
              tma_load_2d(sa, ma, fb, kc, arow);
            } else {
              tma_load_2d(sa, ma, fb, arow, kc);
              tma_load_2d(sa + 8192, ma, fb, arow + 64, kc);
            }
            if (!B_MN) {
              tma_load_2d(sb, mb, fb, kc, brow);
            } else {
#pragma unroll
              for (int j = 0; j < BNH / 64; ++j)
                tma_load_2d(sb + 8192 * j, mb, fb, brow + 64 * j, kc);
            }
          } else {
            // both CTAs' bytes complete on the leader's full barrier, which the
            // leader's producer arms with the pair's total
            const uint32_t fbl = mapa_shared(fb, 0);
            if (crank == 0) mbar_expect_tx(fb, 2 * C::STAGE);
            if (!A_MN) {
              tma_load_2d_pair(sa, ma, fbl, kc, arow);
            } else {
              tma_load_2d_pair(sa, ma, fbl, arow, kc);
              tma_load_2d_pair(sa + 8192, ma, fbl, arow + 64, kc);
            }
            if (!B_MN) {
              tma_load_2d_pair(sb, mb, fbl, kc, brow);
            } else {
#pragma unroll
              for (int j = 0; j < BNH / 64; ++j)
                tma_load_2d_pair(sb + 8192 * j, mb, fbl, brow + 64 * j, kc);
            }
          }
          pending |= 1u << s;
          parbits = (parbits & ~(1u << s)) | (ph << s);
          if (++s == C::STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      if (!ok && crank == 0) {
        // Abort: let every copy issued land before smem is released (a pair's
        // copies all complete on the leader's barriers; the peer is held by the
        // cluster barrier at the end until then).
        for (int i = 0; i < C::STAGES; ++i)
          if (pending & (1u << i))
            bounded_wait(full0 + 8 * i, (parbits >> i) & 1, args.status, LK_ERR_TIMEOUT_DRAIN,
                         nullptr);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0 && crank == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(BM_T, BN, A_MN, B_MN);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      int local = 0;
      for (int t = t_first; t < T && ok; t += t_step, ++local) {
        const int buf = local & 1;
        const uint32_t use = (uint32_t)(local >> 1);
        const bool tok = CG == 2 ? bounded_wait_cluster(tempty0 + 8 * buf, (use & 1) ^ 1, args.status,
                                                        LK_ERR_TIMEOUT_ACCUM, abort_flag)
                                 : bounded_wait(tempty0 + 8 * buf, (use & 1) ^ 1, args.status,
                                                LK_ERR_TIMEOUT_ACCUM, abort_flag);
        if (!tok) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + buf * BN;
        for (int kb = 0; kb < nk; ++kb) {
          if (!bounded_wait(full0 + 8 * s, ph, args.status, LK_ERR_TIMEOUT_FULL, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = sbase + s * C::STAGE;
          const uint32_t sb = sa + C::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < GEMM_BK / 16; ++kk) {
            const uint64_t ad = A_MN ? make_desc_sw128(sa + kk * 2048, 8192, 1024)
                                     : make_desc_sw128(sa + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? make_desc_sw128(sb + kk * 2048, 8192, 1024)
                                     : make_desc_sw128(sb + kk * 32, 16, 1024);
            if constexpr (CG == 2)
              tc_mma_f16_pair(d, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
            else
              tc_mma_f16(d, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          if constexpr (CG == 2)
            tc_commit_pair_mc(empty0 + 8 * s, 0x3);  // both CTAs' producers may refill the stage
          else
            tc_commit(empty0 + 8 * s);
          if (++s == C::STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
        if (ok) {
          if constexpr (CG == 2)
            tc_commit_pair_mc(tfull0 + 8 * buf, 0x3);
          else
            tc_commit(tfull0 + 8 * buf);
        }
      }
      // Make sure every MMA this thread issued has retired before TMEM is freed.
      if constexpr (CG == 2)
        tc_commit_pair(drain_bar);
      else
        tc_commit(drain_bar);
      bounded_wait(drain_bar, 0, args.status, LK_ERR_TIMEOUT_DRAIN, nullptr);
    }
  } else if (AG && warp >= 6) {
    // ------------------------------------------------------ K16 copy warps
    if constexpr (AG == 1)
      ag_copy_warp(args, (warp - 6) * gridDim.x + blockIdx.x, AG_WARPS * gridDim.x, lane);
    else
      gb_copy_warp<BN, B_MN>(args, (warp - 6) * gridDim.x + blockIdx.x, AG_WARPS * gridDim.x, lane,
                             args.ag_rank, args.ag_world);
  } else {
    // ------------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = (int)crank * GEMM_BM + q * 32 + lane;
    const uint32_t tempty_leader = CG == 2 ? mapa_shared(tempty0, 0) : tempty0;
    int local = 0;
    for (int t = t_first; t < T; t += t_step, ++local) {
      int tm, tn;
      gemm_tile_coords(t, args.tiles_m, args.tiles_n, tm, tn);
      tm = (tm + args.m_rot) % args.tiles_m;
      const int buf = local & 1;
      const uint32_t use = (uint32_t)(local >> 1);
      bool ok = bounded_wait(tfull0 + 8 * buf, use & 1, args.status, LK_ERR_TIMEOUT_ACCUM,
                             abort_flag);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const int row = tm * BM_T + row_in_tile;
      const bool row_ok = row < args.M;
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + buf * BN;
      const float alpha = args.alpha;

      if constexpr (EPI == EPI_SWIGLU) {
        // Tile columns [0,128) are gate j, [128,256) are up j, for j in the
        // tile's 128-wide slice of the intermediate dimension.
        __nv_bfloat16* gu = reinterpret_cast<__nv_bfloat16*>(args.D) + (int64_t)row * args.ldd;
        __nv_bfloat16* hrow = args.H + (int64_t)row * args.ldh;
#pragma unroll 1
        for (int c = 0; c < BN / 64; ++c) {
          uint32_t g[32], u[32];
          tmem_ld32(taddr + c * 32, g);
          tmem_ld32(taddr + BN / 2 + c * 32, u);
          tc_wait_ld();
          if (row_ok) {
            const int gcol = tn * BN + c * 32;
            const int ucol = gcol + BN / 2;
            const int hcol = tn * (BN / 2) + c * 32;
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint32_t pg[4], pu[4], ph[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float g0 = __uint_as_float(g[v * 8 + 2 * e]) * alpha;
                const float g1 = __uint_as_float(g[v * 8 + 2 * e + 1]) * alpha;
                const float u0 = __uint_as_float(u[v * 8 + 2 * e]) * alpha;
                const float u1 = __uint_as_float(u[v * 8 + 2 * e + 1]) * alpha;
                pg[e] = pack_bf16x2(g0, g1);
                pu[e] = pack_bf16x2(u0, u1);
                // h from the rounded gate/up so the backward sees consistent values
                const float2 gr = unpack_bf16x2(pg[e]);
                const float2 ur = unpack_bf16x2(pu[e]);
                ph[e] = pack_bf16x2(silu_f(gr.x) * ur.x, silu_f(gr.y) * ur.y);
              }
              if (gcol + v * 8 < args.N)
                *reinterpret_cast<uint4*>(gu + gcol + v * 8) = make_uint4(pg[0], pg[1], pg[2], pg[3]);
              if (ucol + v * 8 < args.N)
                *reinterpret_cast<uint4*>(gu + ucol + v * 8) = make_uint4(pu[0], pu[1], pu[2], pu[3]);
              if (ucol + v * 8 < args.N)
                *reinterpret_cast<uint4*>(hrow + hcol + v * 8) = make_uint4(ph[0], ph[1], ph[2], ph[3]);
            }
          }
        }
      } else if constexpr (EPI == EPI_REMOTE) {
        // K18: stage 32 rows x 64 columns (bf16) per warp in shared memory
        // (128-byte swizzle), then move it into the owner's receive slot over
        // NVLink: one TMA tile store per 32 x 64 block when the owners' tensor
        // maps are given (double-buffered staging), else whole 128-byte row
        // segments with generic stores (4 rows per warp instruction).
        if (args.rmaps != nullptr) {
          const int grow0 = tm * GEMM_BM + q * 32;
          const int owner = grow0 / args.rs_rows;
          const int ydst = args.rs_rank * args.rs_rows + grow0 - owner * args.rs_rows;
          const CUtensorMap* map = args.rmaps + owner;
#pragma unroll 1
          for (int c = 0; c < BN / 64; ++c) {
            uint8_t* stg = smem + C::STAGES * C::STAGE + 1024 + (q * 2 + (c & 1)) * 4096;
            uint32_t r0[32], r1[32];
            tmem_ld32(taddr + c * 64, r0);
            tmem_ld32(taddr + c * 64 + 32, r1);
            tc_wait_ld();
            if (lane == 0) bulk_wait_read<1>();  // the store that last read this buffer is done with it
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const uint32_t* rr = j < 4 ? r0 + 8 * j : r1 + 8 * (j - 4);
              uint4 pk;
              pk.x = pack_bf16x2(__uint_as_float(rr[0]) * alpha, __uint_as_float(rr[1]) * alpha);
              pk.y = pack_bf16x2(__uint_as_float(rr[2]) * alpha, __uint_as_float(rr[3]) * alpha);
              pk.z = pack_bf16x2(__uint_as_float(rr[4]) * alpha, __uint_as_float(rr[5]) * alpha);
              pk.w = pack_bf16x2(__uint_as_float(rr[6]) * alpha, __uint_as_float(rr[7]) * alpha);
              *reinterpret_cast<uint4*>(stg + lane * 128 + ((j ^ (lane & 7)) * 16)) = pk;
            }
            fence_proxy_async_smem();  // generic smem writes -> visible to the TMA unit
            __syncwarp();
            if (lane == 0 && tn * BN + c * 64 < args.N) {
              tma_store_2d(map, smem_u32(stg), tn * BN + c * 64, ydst);
              bulk_commit();
            }
          }
        } else {
        uint8_t* stg = smem + C::STAGES * C::STAGE + 1024 + q * 4096;
#pragma unroll 1
        for (int c = 0; c < BN / 64; ++c) {
          uint32_t r0[32], r1[32];
          tmem_ld32(taddr + c * 64, r0);
          tmem_ld32(taddr + c * 64 + 32, r1);
          tc_wait_ld();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t* rr = j < 4 ? r0 + 8 * j : r1 + 8 * (j - 4);
            uint4 pk;
            pk.x = pack_bf16x2(__uint_as_float(rr[0]) * alpha, __uint_as_float(rr[1]) * alpha);
            pk.y = pack_bf16x2(__uint_as_float(rr[2]) * alpha, __uint_as_float(rr[3]) * alpha);
            pk.z = pack_bf16x2(__uint_as_float(rr[4]) * alpha, __uint_as_float(rr[5]) * alpha);
            pk.w = pack_bf16x2(__uint_as_float(rr[6]) * alpha, __uint_as_float(rr[7]) * alpha);
            *reinterpret_cast<uint4*>(stg + lane * 128 + ((j ^ (lane & 7)) * 16)) = pk;
          }
          __syncwarp();
#pragma unroll
          for (int it = 0; it < 8; ++it) {
            const int rl = it * 4 + (lane >> 3);
            const int j = lane & 7;
            const uint4 pk = *reinterpret_cast<const uint4*>(stg + rl * 128 + ((j ^ (rl & 7)) * 16));
            const int grow = tm * GEMM_BM + q * 32 + rl;
            const int col = tn * BN + c * 64 + j * 8;
            if (grow < args.M && col < args.N) {
              const int owner = grow / args.rs_rows;
              __nv_bfloat16* drow = reinterpret_cast<__nv_bfloat16*>(args.rptrs[owner]) +
                                    (int64_t)(args.rs_rank * args.rs_rows + grow - owner * args.rs_rows) * args.ldd;
              *reinterpret_cast<uint4*>(drow + col) = pk;
            }
          }
          __syncwarp();
        }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(taddr + c * 32, r);
          tc_wait_ld();
          if (!row_ok) continue;
          const int col0 = tn * BN + c * 32;
          if constexpr (EPI == EPI_SWIGLU_BWD) {
            // columns [col0, col0 + 32) of dh lie in one 128-wide block b: gate
            // at 256 b + j, up at 256 b + 128 + j of the gate|up row
            if (col0 < args.N) {
              const int64_t gcol = (int64_t)(col0 >> 7) * 256 + (col0 & 127);
              const __nv_bfloat16* grow = args.R + (int64_t)row * args.ldr + gcol;
              __nv_bfloat16* drow = reinterpret_cast<__nv_bfloat16*>(args.D) + (int64_t)row * args.ldd + gcol;
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                const uint4 gv = *reinterpret_cast<const uint4*>(grow + v * 8);
                const uint4 uv = *reinterpret_cast<const uint4*>(grow + 128 + v * 8);
                const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
                const uint32_t uw[4] = {uv.x, uv.y, uv.z, uv.w};
                uint32_t dg[4], du[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float2 g = unpack_bf16x2(gw[e]), u = unpack_bf16x2(uw[e]);
                  const float d0 = __uint_as_float(r[v * 8 + 2 * e]) * alpha;
                  const float d1 = __uint_as_float(r[v * 8 + 2 * e + 1]) * alpha;
                  const float s0 = 1.0f / (1.0f + __expf(-g.x)), s1 = 1.0f / (1.0f + __expf(-g.y));
                  dg[e] = pack_bf16x2(d0 * u.x * s0 * (1.f + g.x * (1.f - s0)),
                                      d1 * u.y * s1 * (1.f + g.y * (1.f - s1)));
                  du[e] = pack_bf16x2(d0 * g.x * s0, d1 * g.y * s1);
                }
                *reinterpret_cast<uint4*>(drow + v * 8) = make_uint4(dg[0], dg[1], dg[2], dg[3]);
                *reinterpret_cast<uint4*>(drow + 128 + v * 8) = make_uint4(du[0], du[1], du[2], du[3]);
              }
            }
          } else if constexpr (EPI == EPI_BF16 || EPI == EPI_BF16_RESID || EPI == EPI_BF16_ROPE) {
            __nv_bfloat16* drow = reinterpret_cast<__nv_bfloat16*>(args.D) + (int64_t)row * args.ldd;
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              const int col = col0 + v * 8;
              if (col >= args.N) break;
              float f[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(r[v * 8 + e]) * alpha;
              if constexpr (EPI == EPI_BF16_ROPE) {
                if (col < args.rope_cols) {
                  // interleaved pairs (2i, 2i+1) of the head, angle index i = (col % Dh) / 2 + e
                  const int pos = row % args.rope_seq + args.rope_off;
                  const float2* tb = args.rope_table + (int64_t)pos * (args.rope_dh / 2) + (col % args.rope_dh) / 2;
#pragma unroll
                  for (int e = 0; e < 4; ++e) {
                    const float2 cs = tb[e];
                    const float x0 = f[2 * e], x1 = f[2 * e + 1];
                    f[2 * e] = x0 * cs.x - x1 * cs.y;
                    f[2 * e + 1] = x0 * cs.y + x1 * cs.x;
                  }
                }
              }
              if constexpr (EPI == EPI_BF16_RESID) {
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
                  make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                             pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
            }
          } else {
            float* drow = reinterpret_cast<float*>(args.D) + (int64_t)row * args.ldd;
#pragma unroll
            for (int v = 0; v < 8; ++v) {
              const int col = col0 + v * 4;
              if (col >= args.N) break;
              float4 o = make_float4(__uint_as_float(r[v * 4]) * alpha,
                                     __uint_as_float(r[v * 4 + 1]) * alpha,
                                     __uint_as_float(r[v * 4 + 2]) * alpha,
                                     __uint_as_float(r[v * 4 + 3]) * alpha);
              if constexpr (EPI == EPI_F32_ACC) {
                const float4 old = *reinterpret_cast<const float4*>(drow + col);
                o.x += old.x;
                o.y += old.y;
                o.z += old.z;
                o.w += old.w;
              }
              *reinterpret_cast<float4*>(drow + col) = o;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (CG == 2)
          mbar_arrive_cluster(tempty_leader + 8 * buf);
        else
          mbar_arrive(tempty0 + 8 * buf);
      }
    }
    if constexpr (EPI == EPI_REMOTE) {
      if (lane == 0) bulk_wait<0>();  // every TMA store of this warp has landed in peer memory
      __syncwarp();
    }
  }

  tc_fence_before();
  if constexpr (CG == 2)
    cluster_sync();  // the pair's MMAs, copies and TMEM reads are all done
  else
    __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (CG == 2)
      tmem_dealloc_pair(tmem, C::TMEM_COLS);
    else
      tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <int BN, bool A_MN, bool B_MN, int EPI, int AG = 0, int CG = 1>
int launch_gemm(const LkGemmDesc& g, cudaStream_t stream) {
  using C = GemmCfg<BN, CG>;
  GemmArgs args{};
  args.M = g.M;
  args.N = g.N;
  args.K = g.K;
  args.D = g.d;
  args.ldd = g.ldd;
  args.R = reinterpret_cast<const __nv_bfloat16*>(g.r);
  args.ldr = g.ldr;
  args.H = reinterpret_cast<__nv_bfloat16*>(g.h);
  args.ldh = g.ldh;
  args.alpha = g.alpha;
  args.status = g.status;
  args.tiles_m = cdiv(g.M, GEMM_BM * CG);
  args.tiles_n = cdiv(g.N, BN);
  CUtensorMap ta, tb, ta2, tb2;
  const CUtensorMapDataType bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  if (!make_tmap_2d(&ta, g.a, bf, 2, g.a_rows, g.a_cols, g.a_ld, A_MN ? 64 : GEMM_BM, 64)) return -1;
  if (!make_tmap_2d(&tb, g.b, bf, 2, g.b_rows, g.b_cols, g.b_ld, B_MN ? 64 : BN / CG, 64)) return -1;
  args.K2 = g.K2;
  if (g.K2 > 0) {
    if (!make_tmap_2d(&ta2, g.a2, bf, 2, g.a2_rows, g.a2_cols, g.a2_ld, A_MN ? 64 : GEMM_BM, 64)) return -1;
    if (!make_tmap_2d(&tb2, g.b2, bf, 2, g.b2_rows, g.b2_cols, g.b2_ld, B_MN ? 64 : BN / CG, 64)) return -1;
  } else {
    ta2 = ta;
    tb2 = tb;
  }
  args.m_rot = g.m_rot;
  args.rptrs = reinterpret_cast<void* const*>(g.rptrs);
  args.rmaps = reinterpret_cast<const CUtensorMap*>(g.rmaps);
  args.rs_rows = g.rs_rows;
  args.rs_rank = g.rs_rank;
  args.ag_src = reinterpret_cast<const uint8_t* const*>(g.ag_src);
  args.ag_ld_src = g.ag_ld_src;
  args.ag_ld_dst = g.a_ld * 2;
  args.ag_dst = reinterpret_cast<uint8_t*>(const_cast<void*>(g.a));
  args.ag_rows = g.ag_rows;
  args.ag_rank = g.ag_rank;
  args.ag_world = g.ag_world;
  args.ag_row_bytes = (int)(g.a_cols * 2);
  args.ag_count = g.ag_count;
  args.gb_src = reinterpret_cast<const uint8_t* const*>(g.gb_src);
  args.gb_chunk = g.gb_chunk;
  args.gb_len = g.gb_len;
  args.gb_boff = g.gb_boff;
  args.gb_dst = reinterpret_cast<uint8_t*>(g.gb_dst);
  args.gb_count = g.gb_count;
  args.rope_table = reinterpret_cast<const float2*>(g.rope_table);
  args.rope_cols = g.rope_cols;
  args.rope_dh = g.rope_dh > 0 ? g.rope_dh : 64;
  args.rope_seq = g.rope_seq > 0 ? g.rope_seq : (1 << 30);
  args.rope_off = g.rope_off;
  auto kern = gemm_tc_kernel<BN, A_MN, B_MN, EPI, AG, CG>;
  static uint64_t attr_set = 0;  // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  // K18 staging: 1024-aligned after the barriers, 2 x 4 KB per epilogue warp
  constexpr int SMEM = C::SMEM + (EPI == EPI_REMOTE ? 1024 - C::BAR_BYTES + 8 * 4096 : 0);
  if (!(attr_set & (1ull << dev))) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    attr_set |= 1ull << dev;
  }
  const int tiles = args.tiles_m * args.tiles_n;
  if constexpr (CG == 2) {
    // one cluster (CTA pair) per two SMs, persistent over the 256 x BN tiles
    const int pairs = tiles < num_sms() / 2 ? tiles : num_sms() / 2;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(GEMM_THREADS);
    cfg.dynamicSmemBytes = SMEM;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, ta2, tb2, args);
    if (e != cudaSuccess) {
      last_error() = std::string("gemm pair launch: ") + cudaGetErrorString(e);
      return -1;
    }
    return check_launch("gemm_tc_kernel_pair");
  }
  const int grid = tiles < num_sms() ? tiles : num_sms();
  if constexpr (AG != 0) {
    // CTAs wait on data copied by other CTAs: they must all be resident
    int* cnt = AG == 1 ? g.ag_count : g.gb_count;
    const int ncnt = AG == 1 ? args.tiles_m : args.tiles_n;
    if (cudaMemsetAsync(cnt, 0, sizeof(int) * ncnt, stream) != cudaSuccess) return fail("gemm_ag: memset failed");
    void* params[] = {&ta, &tb, &ta2, &tb2, &args};
    cudaError_t e = cudaLaunchCooperativeKernel((void*)kern, dim3(grid), dim3(GEMM_THREADS + 32 * AG_WARPS), params,
                                                SMEM, stream);
    if (e != cudaSuccess) {
      last_error() = std::string("gemm_ag cooperative launch: ") + cudaGetErrorString(e);
      return -1;
    }
    return check_launch("gemm_tc_kernel_ag");
  } else {
    kern<<<grid, GEMM_THREADS, SMEM, stream>>>(ta, tb, ta2, tb2, args);
    return check_launch("gemm_tc_kernel");
  }
}

// CTA-pair policy (gemm_dispatch.cu): mode 0 off, 1 on where applicable.
int& gemm_pair_mode();
bool use_pair(const LkGemmDesc& g);

// Per-epilogue dispatchers (each defined in its own translation unit).
int gemm_dispatch_bf16(const LkGemmDesc& g, cudaStream_t s);
int gemm_dispatch_f32(const LkGemmDesc& g, cudaStream_t s);
int gemm_dispatch_fused(const LkGemmDesc& g, cudaStream_t s);
int gemm_dispatch_comm(const LkGemmDesc& g, cudaStream_t s);

}  // namespace lk
