// Prefill det linear on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// Y[s, n] = requantize(sum_k X[s, k] * W[n, k])   (wrapping i64 sum; the
// arithmetic of linear_into / matmul_det in the reference's det path)
//
// Exact integer decomposition.  With X_u = X + 2^e (u32; e = 31, or e = 23
// for an activation row whose values all lie in [-2^23, 2^23), so that its
// X_u < 2^24 and byte limb 3 is zero) and W_u = W + 2^15 (u16), both
// non-negative,
//   sum_k X W = sum_k X_u W_u - 2^15 sum_k X_u - 2^e sum_k W_u + 2^(15+e) K
// holds exactly in wrapping i64.  X_u splits into four byte limbs x_a and W_u
// into two byte limbs w_b (all u8), and
//   sum_k X_u W_u = sum_{a,b} 2^(8(a+b)) P_ab,   P_ab = sum_k x_a w_b.
// Each P_ab is an unsigned int8 tensor-core product accumulated in 32 bits.
//
// One MMA per activation limb: the B operand stacks the low-byte plane rows
// of an N tile (96 weight rows) above the high-byte plane rows (N = 192), so
// MMA a writes [P_a0 | P_a1] into TMEM columns [96a, 96a + 192).  The four
// regions overlap by 96 columns: column block g = [96g, 96g + 96) accumulates
// exactly the products with shift 8g (P_g0 + P_(g-1)1), 480 columns in all.
// A block holds at most two non-negative products of at most 255*255*K each,
// so its 32-bit accumulator is exact (read as u32) for K < 33025.  The
// epilogue recombines the five blocks and the two row-sum corrections in
// wrapping i64 and requantizes: bit-exact with the CUDA-core linear.
//
// Pipeline (persistent CTAs, output tiles of 128 tokens x 96 weight rows):
// warp 8 streams activation limb tiles (4 x 128 x 64 B) and the stacked
// weight tile (192 x 64 B) with TMA (tiled, 64-byte swizzle, each CTA loading
// its own tiles) into a 4-stage ring that runs across tile boundaries; warp 9
// issues the MMAs (M=128, N=192, K=32, kind::i8, u8 x u8 -> s32) and frees
// stages with tcgen05.commit; warps 0-7 drain the accumulator through
// tcgen05.ld into a shared-memory tile, release TMEM, then finish the
// epilogue and store while the next tile's MMAs run.  Every mbarrier wait is
// bounded and reports a timeout through the library's pipeline error flag.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "det_dev.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

namespace rdet {

// set when a bounded pipeline wait gives up (read by tc_error_flag)
__device__ int g_tc_err = 0;
// the CTA-pair GEMM for prompts of more than 128 tokens (0: one-CTA tiles;
// RDET_TC_PAIR=0 in the environment selects them)
static bool g_tc_pair = [] {
  const char* e = getenv("RDET_TC_PAIR");
  return !(e && e[0] == '0');
}();

namespace {

constexpr int kTcM = 128;         // output rows (tokens) per tile
constexpr int kTcN = 96;          // output columns (weight rows) per tile
constexpr int kTcNB = 2 * kTcN;   // stacked B rows (low and high byte planes)
constexpr int kTcKB = 64;         // K bytes per stage (one 64-byte swizzle row)
constexpr int kTcStages = 4;
constexpr int kTcATile = kTcM * kTcKB;         // 8 KB per activation limb
constexpr int kTcBTile = kTcNB * kTcKB;        // 12 KB
constexpr int kTcStage = 4 * kTcATile + kTcBTile;  // 44 KB
constexpr int kTcOutStride = kTcN + 1;                 // staged output row (odd: conflict-free)
constexpr int kTcStageOut = kTcM * kTcOutStride * 4;   // 49.7 KB output staging
constexpr int kTcSmem = kTcStages * kTcStage + kTcStageOut + 1024;  // + alignment slack
constexpr int kTcEpiWarps = 8;  // two per TMEM lane quarter, each half of the columns
constexpr int kTcThreads = 32 * (kTcEpiWarps + 2);
constexpr uint32_t kTcCols = 512;  // TMEM columns allocated (480 used)
constexpr int kT2Mrows = 256;      // tokens per CTA-pair tile
constexpr uint64_t kRowOff23 = 1ull << 63;  // row-sum flag: the row's offset is 2^23, not 2^31

// An activation row's corrections.  Its planes hold X + 2^e (e = 23 when the
// row sum's top bit is set, else 31), so for one output
//   sum X W = sum X_u W_u - 2^15 sum X_u - 2^e sum W_u + 2^(15 + e) K.
// row_corr = 2^15 sum X_u - 2^(15 + e) K (wrapping); the weight term is
// brow << e.
struct RowCorr {
  uint64_t corr;
  uint32_t e;
};
__device__ __forceinline__ RowCorr row_corr(uint64_t rw, int K) {
  RowCorr r;
  r.e = (rw & kRowOff23) ? 23u : 31u;
  r.corr = ((rw & ~kRowOff23) << 15) - ((uint64_t)K << (15 + r.e));
  return r;
}

using namespace tcx;

// sum over g of blk[g] * 2^(8g): the overlapping TMEM column blocks of one
// output (each block a u32 accumulator)
__device__ __forceinline__ uint64_t limb_sum(uint32_t g0, uint32_t g1, uint32_t g2, uint32_t g3, uint32_t g4) {
  return (uint64_t)g0 + ((uint64_t)g1 << 8) + ((uint64_t)g2 << 16) + ((uint64_t)g3 << 24) + ((uint64_t)g4 << 32);
}

// kind::i8 instruction descriptors of this file's MMAs (M = 128)
constexpr uint32_t kTcIdesc = idesc_u8(kTcNB);    // both byte planes
constexpr uint32_t kTcIdescHalf = idesc_u8(kTcN); // one byte plane

// ---------------------------------------------------------------------------
// operand preparation
// ---------------------------------------------------------------------------

// Activation rows -> four byte planes of X + 2^e and the row sums of X + 2^e,
// e chosen per row: 23 when every value of the row lies in [-2^23, 2^23) (then
// X + 2^23 < 2^24 and limb 3 is zero), else 31.  The row sum carries the choice
// in its top bit (set for 23; a sum is below 2^47); tile4[row / 256] is set
// when a row of that 256-row tile needs the fourth limb (tile4 starts at 0).
__global__ void tc_act_prep_kernel(const int32_t* __restrict__ X, int S, int K, uint8_t* __restrict__ planes,
                                   uint64_t* __restrict__ rowsum, uint32_t* __restrict__ tile4) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int s = blockIdx.x;
  const int4* xr = reinterpret_cast<const int4*>(X + (size_t)s * K);
  const size_t plane = (size_t)S * K;
  int wide = 0;
  for (int c = threadIdx.x; c < K / 4 && !wide; c += blockDim.x) {
    const int4 v = xr[c];
    wide |= (v.x < -(1 << 23) || v.x >= (1 << 23) || v.y < -(1 << 23) || v.y >= (1 << 23) || v.z < -(1 << 23) ||
             v.z >= (1 << 23) || v.w < -(1 << 23) || v.w >= (1 << 23));
  }
  const bool four = __syncthreads_or(wide) != 0;
  const uint32_t off = four ? 0x80000000u : 0x00800000u;
  uint64_t sum = 0;
  for (int c = threadIdx.x; c < K / 4; c += blockDim.x) {
    const int4 v = xr[c];
    const uint32_t u[4] = {(uint32_t)v.x + off, (uint32_t)v.y + off, (uint32_t)v.z + off, (uint32_t)v.w + off};
    sum += (uint64_t)u[0] + u[1] + u[2] + u[3];
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const uint32_t packed = ((u[0] >> (8 * a)) & 0xffu) | (((u[1] >> (8 * a)) & 0xffu) << 8) |
                              (((u[2] >> (8 * a)) & 0xffu) << 16) | (((u[3] >> (8 * a)) & 0xffu) << 24);
      *reinterpret_cast<uint32_t*>(planes + a * plane + (size_t)s * K + 4 * c) = packed;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  __shared__ uint64_t part[32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint64_t t = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += part[w];
    rowsum[s] = four ? t : (t | kRowOff23);
    if (four && tile4) atomicOr(&tile4[s / kT2Mrows], 1u);
  }
}

// Weight rows (i16) -> low/high byte planes of W + 2^15 and their row sums.
// Plane row R maps to source row R, or for a gate/up pair to gate row
// 48*(R/96) + R%96 (R%96 < 48) or up row 48*(R/96) + R%96 - 48.
// A slice takes source rows [row0, row0 + rows) and columns [col0, col0 + K)
// of a matrix with row stride ld.
__global__ void tc_weight_prep_kernel(const int16_t* __restrict__ W, const int16_t* __restrict__ U, int rows,
                                      int K, size_t plane, uint8_t* __restrict__ planes, uint64_t* __restrict__ rowsum,
                                      int row0, int col0, int ld) {
  const int R = blockIdx.x;
  const int16_t* src = nullptr;
  if (U == nullptr) {
    if (R < rows) src = W + (size_t)(row0 + R) * ld + col0;
  } else {
    const int b = R / kTcN, j = R % kTcN, h = kTcN / 2;
    const int r = b * h + (j < h ? j : j - h);
    if (r < rows) src = (j < h ? W : U) + (size_t)(row0 + r) * ld + col0;
  }
  uint64_t sum = 0;
  for (int c = threadIdx.x; c < K / 8; c += blockDim.x) {
    uint16_t u[8];
    if (src) {
      const int4 v = reinterpret_cast<const int4*>(src)[c];
      const int16_t* e = reinterpret_cast<const int16_t*>(&v);
#pragma unroll
      for (int i = 0; i < 8; ++i) u[i] = (uint16_t)((int32_t)e[i] + 32768);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) u[i] = 0;
    }
    uint64_t lo = 0, hi = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      sum += u[i];
      lo |= (uint64_t)(u[i] & 0xffu) << (8 * i);
      hi |= (uint64_t)(u[i] >> 8) << (8 * i);
    }
    *reinterpret_cast<uint64_t*>(planes + (size_t)R * K + 8 * c) = lo;
    *reinterpret_cast<uint64_t*>(planes + plane + (size_t)R * K + 8 * c) = hi;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  __shared__ uint64_t part[32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint64_t t = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += part[w];
    rowsum[R] = t;
  }
}

// ---------------------------------------------------------------------------
// the GEMM
// ---------------------------------------------------------------------------
// EPI: 0 plain, 1 gelu(y) * vec[s, n], 2 gate/up pair (gelu(gate) * up)
//
// Persistent: CTA b takes tiles b, b + grid, ... (N tile fastest).  The
// producer streams stages across tile boundaries, so the next tile's first
// stages load while the epilogue drains the previous accumulator; the MMA
// warp starts a tile once the epilogue has moved the accumulator out of TMEM
// (tmem_empty).  No zeroing: the first K step of a tile writes every TMEM
// column once with accumulate off before anything accumulates into it
// (limbs 0 and 2 fresh, limb 1 onto them, limb 3 split into its low-plane
// half that accumulates and its high-plane half that is fresh).
// EPI 3 (split K): work item i is tile i / ks, K range i % ks of ks equal
// parts; the epilogue writes the raw sum of the range, sum_g 2^(8g) G_g (no
// corrections, not requantized), to part[(i % ks)][S][nrows] and
// tc_splitk_reduce finishes the output.
template <int EPI>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_linear_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap,
                     const uint64_t* __restrict__ arow, const uint64_t* __restrict__ brow, int S, int N, int K,
                     int ntiles_n, int ntiles, int ks, int nrows, int32_t* __restrict__ Y,
                     const int32_t* __restrict__ vec, int ldv, uint64_t* __restrict__ part) {
  extern __shared__ __align__(16) unsigned char tc_smem_raw[];
  __shared__ __align__(8) uint64_t full[kTcStages], empty[kTcStages], accf, tmem_empty;
  __shared__ uint32_t tmem_holder;
  __shared__ int fail;
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~(uintptr_t)1023);
  int32_t* stage_out = reinterpret_cast<int32_t*>(smem + (size_t)kTcStages * kTcStage);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = (K + kTcKB - 1) / kTcKB;
  const int nitems = ntiles * ks;  // ks == 1 except in split-K mode
  const int my_tiles = blockIdx.x < nitems ? (nitems - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (threadIdx.x == 0) {
    for (int i = 0; i < kTcStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(&accf, 1);
    mbar_init(&tmem_empty, kTcEpiWarps);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fail = 0;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_holder)),
                 "r"(kTcCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = tmem_holder;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (warp == kTcEpiWarps) {
    // ---- producer: every stage of every tile of this CTA, through the ring
    if (lane == 0) {
      int q = 0;
      for (int it = 0; it < my_tiles; ++it) {
        const int item = blockIdx.x + it * gridDim.x, t = item / ks, sp = item % ks;
        const int m0 = (t / ntiles_n) * kTcM, r0 = (t % ntiles_n) * kTcN;
        const int kb0 = (int)((int64_t)nkb * sp / ks), kb1 = (int)((int64_t)nkb * (sp + 1) / ks);
        for (int kb = kb0; kb < kb1; ++kb, ++q) {
          const int st = q % kTcStages;
          if (q >= kTcStages && !mbar_wait(&empty[st], ((q / kTcStages) - 1) & 1)) fail = 1;
          unsigned char* sbuf = smem + (size_t)st * kTcStage;
          mbar_expect_tx(&full[st], kTcStage);
          for (int a = 0; a < 4; ++a) tma_load_3d(sbuf + a * kTcATile, &amap, kb * kTcKB, m0, a, &full[st]);
          tma_load_3d(sbuf + 4 * kTcATile, &bmap, kb * kTcKB, r0, 0, &full[st]);
          tma_load_3d(sbuf + 4 * kTcATile + kTcN * kTcKB, &bmap, kb * kTcKB, r0, 1, &full[st]);
        }
      }
    }
  } else if (warp == kTcEpiWarps + 1) {
    // ---- MMA issue
    if (lane == 0) {
      int q = 0, qlast = 0;
      for (int it = 0; it < my_tiles; ++it) {
        const int sp = (blockIdx.x + it * gridDim.x) % ks;
        qlast += (int)((int64_t)nkb * (sp + 1) / ks) - (int)((int64_t)nkb * sp / ks);
      }
      for (int it = 0; it < my_tiles; ++it) {
        const int sp = (blockIdx.x + it * gridDim.x) % ks;
        const int kb0 = (int)((int64_t)nkb * sp / ks), kb1 = (int)((int64_t)nkb * (sp + 1) / ks);
        if (it > 0 && !mbar_wait(&tmem_empty, (it - 1) & 1)) fail = 1;
        fence_after();
        for (int kb = kb0; kb < kb1; ++kb, ++q) {
          const int st = q % kTcStages;
          if (!mbar_wait(&full[st], (q / kTcStages) & 1)) fail = 1;
          fence_after();
          const unsigned char* sbuf = smem + (size_t)st * kTcStage;
          const uint32_t baddr = su32(sbuf + 4 * kTcATile);
#pragma unroll
          for (int j = 0; j < kTcKB / 32; ++j) {
            const uint64_t bdesc = smem_desc_sw64(baddr + 32 * j);
            const uint64_t ad[4] = {smem_desc_sw64(su32(sbuf) + 32 * j), smem_desc_sw64(su32(sbuf + kTcATile) + 32 * j),
                                    smem_desc_sw64(su32(sbuf + 2 * kTcATile) + 32 * j),
                                    smem_desc_sw64(su32(sbuf + 3 * kTcATile) + 32 * j)};
            if (kb == kb0 && j == 0) {
              mma_i8(tmem + 0 * kTcN, ad[0], bdesc, kTcIdesc, 0u);
              mma_i8(tmem + 2 * kTcN, ad[2], bdesc, kTcIdesc, 0u);
              mma_i8(tmem + 1 * kTcN, ad[1], bdesc, kTcIdesc, 1u);
              mma_i8(tmem + 3 * kTcN, ad[3], bdesc, kTcIdescHalf, 1u);
              mma_i8(tmem + 4 * kTcN, ad[3], smem_desc_sw64(baddr + kTcN * kTcKB), kTcIdescHalf, 0u);
            } else {
#pragma unroll
              for (int a = 0; a < 4; ++a) mma_i8(tmem + (uint32_t)(kTcN * a), ad[a], bdesc, kTcIdesc, 1u);
            }
          }
          // free the stage once these MMAs have read it (the CTA's last stages
          // are never reloaded, so nothing waits for them)
          if (q + kTcStages < qlast) mma_commit(&empty[st]);
        }
        mma_commit(&accf);
      }
    }
  } else {
    // ---- epilogue: warp w reads TMEM lanes 32*(w%4).. and column half w/4
    constexpr int kOut = EPI == 2 ? kTcN / 2 : kTcN;  // outputs per tile row
    constexpr int kHalf = kOut / 2;
    const int quarter = warp & 3, half = warp >> 2;
    const int rl = 32 * quarter + lane;
    const uint32_t tbase = tmem + ((uint32_t)(32 * quarter) << 16);
    for (int it = 0; it < my_tiles; ++it) {
      const int item = blockIdx.x + it * gridDim.x, t = item / ks, sp = item % ks;
      const int m0 = (t / ntiles_n) * kTcM, nt = t % ntiles_n, r0 = nt * kTcN;
      const int nbase = EPI == 2 ? nt * (kTcN / 2) : r0;
      const int m = m0 + rl;
      const bool mrow = m < S;
      const RowCorr rc = row_corr(mrow ? arow[m] : 0, K);
      if (!mbar_wait(&accf, it & 1)) fail = 1;
      fence_after();
      if (EPI == 3) {
        // raw partial of this K range for all 96 plane rows, straight from registers
        for (int c0 = half * (kTcN / 2); c0 < (half + 1) * (kTcN / 2); c0 += 8) {
          uint32_t g[5][8];
#pragma unroll
          for (int gg = 0; gg < 5; ++gg) tmem_ld8(tbase + kTcN * gg + c0, g[gg]);
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
          if (mrow) {
            uint64_t* dst = part + ((size_t)sp * S + m) * nrows + r0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int j = c0 + i;
              if (r0 + j < nrows)
                dst[j] = limb_sum(g[0][i], g[1][i], g[2][i], g[3][i], g[4][i]);
            }
          }
        }
        fence_before();
        __syncwarp();
        if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(&tmem_empty)) : "memory");
        continue;
      }
      if constexpr (EPI != 3) {
      // phase 1, TMEM held: recombine, correct and requantize 16 plane rows
      // per TMEM wait into this thread's staging row (a gate/up pair stages
      // gate at column j and up at column kTcN / 2 + j)
      constexpr int kStep = EPI == 2 ? 8 : 16;
      for (int c0 = half * kHalf; c0 < (half + 1) * kHalf; c0 += kStep) {
        uint32_t g[5][2][8];
#pragma unroll
        for (int gg = 0; gg < 5; ++gg) {
          tmem_ld8(tbase + kTcN * gg + c0, g[gg][0]);
          tmem_ld8(tbase + kTcN * gg + (EPI == 2 ? kTcN / 2 : 8) + c0, g[gg][1]);
        }
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int pr = c0 + (EPI == 2 ? (i >> 3) * (kTcN / 2) + (i & 7) : i);  // plane row in the tile
          const int n = nbase + c0 + (EPI == 2 ? (i & 7) : i);
          int32_t y = 0;
          // plane rows of a pair cover whole tiles; a plain matrix has N rows
          if (mrow && n < N) {
            uint64_t acc = limb_sum(g[0][i >> 3][i & 7], g[1][i >> 3][i & 7], g[2][i >> 3][i & 7],
                                    g[3][i >> 3][i & 7], g[4][i >> 3][i & 7]);
            acc -= rc.corr + (brow[r0 + pr] << rc.e);
            y = requantize((int64_t)acc);
          }
          stage_out[rl * kTcOutStride + pr] = y;
        }
      }
      // the accumulator is in shared memory: TMEM is free for the next tile
      fence_before();
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(&tmem_empty)) : "memory");
      // phase 2, overlapping the next tile's MMAs: the GELU epilogues on this
      // thread's own staged values
      if constexpr (EPI == 1 || EPI == 2) {
        if (mrow) {
          for (int j = half * kHalf; j < (half + 1) * kHalf; ++j) {
            const int n = nbase + j;
            if (n >= N) break;
            int32_t* sp_ = &stage_out[rl * kTcOutStride + j];
            *sp_ = mul_sat(gelu_act(*sp_), EPI == 2 ? sp_[kTcN / 2] : vec[(size_t)m * ldv + n]);
          }
        }
      }
      asm volatile("bar.sync 1, %0;" ::"n"(32 * kTcEpiWarps) : "memory");  // staging complete
      for (int r = warp; r < kTcM; r += kTcEpiWarps) {
        const int mm = m0 + r;
        if (mm >= S) break;
        for (int c = lane; c < kOut; c += 32) {
          const int n = nbase + c;
          if (n < N) Y[(size_t)mm * N + n] = stage_out[r * kTcOutStride + c];
        }
      }
      asm volatile("bar.sync 1, %0;" ::"n"(32 * kTcEpiWarps) : "memory");  // staging free again
      }
    }
  }
  fence_before();
  __syncthreads();
  if (fail && threadIdx.x == 0) atomicExch(&g_tc_err, 1);
  if (warp == 0) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcCols) : "memory");
  }
}

// ---------------------------------------------------------------------------
// The same GEMM on a CTA pair (tcgen05 cta_group::2, a cluster of two CTAs):
// an output tile is 256 tokens x 96 weight rows.  CTA r of the pair holds
// tokens [m0 + 128r, m0 + 128r + 128) of the four activation limbs (the A
// rows of its half of M = 256) and byte plane r of the tile's 96 weight rows
// (its half of the B operand's N = 192 rows: plane 0 in CTA 0, plane 1 in
// CTA 1).  Every MMA therefore reads 4 KB of A and 3 KB of B from each SM's
// shared memory instead of 4 KB and 6 KB, and a stage moves 38 KB per SM
// instead of 44 KB.  The MMA's N columns keep the one-CTA order (low plane,
// then high plane), so the TMEM blocks and the epilogue are those of
// tc_linear_kernel, each CTA draining its own 128 rows.
// The leader (rank 0) issues every MMA; both CTAs' TMA loads (cta_group::2,
// no multicast) signal the leader's stage barrier, which expects both
// halves' bytes; the leader's commits arrive on both CTAs' barriers; both
// epilogues release TMEM on the leader's barrier.  Block 4 (shift 32) is
// zeroed by the epilogue before each tile (a plane cannot be addressed alone
// when B is split by plane across the pair), so a tile's first K step runs
// limbs 0 and 2 with accumulate off and limbs 1 and 3 onto them.  A tile whose
// 256 rows all have e = 23 loads and multiplies activation limbs 0-2 only (6
// limb products instead of 8; block 4 stays zero).
// Tiles go round the pairs in the order that keeps the smaller operand in L2
// (m_fast: all token tiles of a weight tile before the next weight tile).
// ---------------------------------------------------------------------------
constexpr int kT2M = kT2Mrows;                     // tokens per pair tile
static_assert(kT2M == kTcFlagRows, "one tile flag per pair tile");
static_assert(kT2M == 2 * kTcM, "a pair tile is two one-CTA tiles");
// The TMA ring: four 38 KB stages (four activation limbs and a weight plane),
// or five 30 KB stages when no tile of the launch needs the fourth limb.  The
// loads' latency, not L2 bandwidth, bounds the main loop, so the bytes in
// flight set its speed.
constexpr int kT2Stages = 4;
constexpr int kT2Stages3 = 5;
constexpr int kT2BTile = kTcN * kTcKB;             // 6 KB: one weight plane
constexpr int kT2Stage = 4 * kTcATile + kT2BTile;  // 38 KB
constexpr int kT2Stage3 = 3 * kTcATile + kT2BTile; // 30 KB
static_assert(kT2Stages3 * kT2Stage3 <= kT2Stages * kT2Stage, "both rings fit the same shared memory");
static_assert(kT2Stage3 % 1024 == 0, "stages keep the swizzle alignment");
constexpr int kT2Smem = kT2Stages * kT2Stage + kTcStageOut + 1024;
// kind::i8 instruction descriptor with M = 256 (cta_group::2), N = 192
constexpr uint32_t kT2Idesc = (2u << 4) | ((uint32_t)(kTcNB >> 3) << 17) | ((uint32_t)(kT2M >> 4) << 24);

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same location in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// tiled 3D TMA load into this CTA's shared memory whose completion is counted
// on an mbarrier of either CTA of the pair (no multicast)
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map, int x, int y, int z,
                                                 uint32_t bar_cluster, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
      "[%1, {%2, %3, %4}], [%5], %6;" ::"r"(su32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar_cluster), "l"(policy)
      : "memory");
}
// L2 policies: the operand every tile of a wave re-reads stays (evict_last),
// the one read once streams through (evict_first)
__device__ __forceinline__ uint64_t l2_policy(bool keep) {
  uint64_t p;
  if (keep) asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  else asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void mma_i8_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// arrive on the barrier at the same offset in both CTAs once the MMAs issued
// so far have completed
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          su32(bar)),
      "h"((uint16_t)3)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
__device__ __forceinline__ void tmem_st8_zero(uint32_t taddr) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(taddr), "r"(0)
               : "memory");
}

template <int EPI>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_linear2_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap,
                      const uint64_t* __restrict__ arow, const uint64_t* __restrict__ brow, int S, int N, int K,
                      int ntiles_m, int ntiles_n, int m_fast, int32_t* __restrict__ Y,
                      const int32_t* __restrict__ vec, int ldv, const uint32_t* __restrict__ tile4) {
  extern __shared__ __align__(16) unsigned char tc_smem_raw[];
  __shared__ __align__(8) uint64_t full[kT2Stages3], empty[kT2Stages3], accf, tmem_empty;
  __shared__ uint32_t tmem_holder;
  __shared__ int fail;
  // each epilogue warp's copy of the tile's weight row sums, shifted by 23
  // (first half) and by 31 (second half): the row's e picks one
  __shared__ uint64_t bsum[kTcEpiWarps][2 * kTcN];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~(uintptr_t)1023);
  int32_t* stage_out = reinterpret_cast<int32_t*>(smem + (size_t)kT2Stages * kT2Stage);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int nkb = (K + kTcKB - 1) / kTcKB;
  const int ntiles = ntiles_m * ntiles_n;
  const int my_tiles = pair < ntiles ? (ntiles - 1 - pair) / npairs + 1 : 0;
  auto tile_of = [&](int it, int& m0, int& nt) {
    const int t = pair + it * npairs;
    const int mt = m_fast ? t % ntiles_m : t / ntiles_n;
    nt = m_fast ? t / ntiles_m : t % ntiles_n;
    m0 = mt * kT2M;
  };
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (threadIdx.x == 0) {
    for (int i = 0; i < kT2Stages3; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(&accf, 1);
    mbar_init(&tmem_empty, 2 * kTcEpiWarps);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fail = 0;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_holder)),
                 "r"(kTcCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers initialised and TMEM allocated
  fence_after();
  const uint32_t tmem = tmem_holder;
  const uint32_t tmem_empty_leader = mapa_rank(su32(&tmem_empty), 0);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // ring shape (every thread derives the same one from the tile flags)
  bool any4 = tile4 == nullptr;
  for (int i = 0; i < ntiles_m && !any4; ++i) any4 = tile4[i] != 0;
  const int nst = any4 ? kT2Stages : kT2Stages3;
  const int stage_bytes = any4 ? kT2Stage : kT2Stage3;
  const int boff = (any4 ? 4 : 3) * kTcATile;  // the weight plane's offset in a stage
  if (warp == kTcEpiWarps) {
    // ---- producer (both CTAs): this CTA's A rows and weight plane, counted
    // on the leader's stage barrier
    if (lane == 0) {
      // m_fast: the activation tiles are re-read by every weight tile
      const uint64_t pol_a = l2_policy(m_fast != 0), pol_b = l2_policy(m_fast == 0);
      int q = 0, st = 0;
      uint32_t ph = 0;  // parity of the ring round
      for (int it = 0; it < my_tiles; ++it) {
        int m0, nt;
        tile_of(it, m0, nt);
        // a tile whose rows all fit 24 bits skips activation limb 3 (zero)
        const int limbs = (tile4 == nullptr || tile4[m0 / kT2M]) ? 4 : 3;
        const uint32_t tx = 2u * (uint32_t)(limbs * kTcATile + kT2BTile);
        for (int kb = 0; kb < nkb; ++kb, ++q) {
          if (q >= nst && !mbar_wait(&empty[st], ph ^ 1u)) fail = 1;
          unsigned char* sbuf = smem + (size_t)st * stage_bytes;
          if (rank == 0) mbar_expect_tx(&full[st], tx);
          const uint32_t bar = mapa_rank(su32(&full[st]), 0);
          for (int a = 0; a < limbs; ++a)
            tma_load_3d_pair(sbuf + a * kTcATile, &amap, kb * kTcKB, m0 + kTcM * (int)rank, a, bar, pol_a);
          tma_load_3d_pair(sbuf + boff, &bmap, kb * kTcKB, nt * kTcN, (int)rank, bar, pol_b);
          if (++st == nst) { st = 0; ph ^= 1u; }
        }
      }
    }
  } else if (warp == kTcEpiWarps + 1) {
    // ---- MMA issue (leader only)
    if (rank == 0 && lane == 0) {
      const int qlast = my_tiles * nkb;
      int q = 0, st = 0;
      uint32_t ph = 0;  // parity of the ring round
      for (int it = 0; it < my_tiles; ++it) {
        int m0, nt;
        tile_of(it, m0, nt);
        const bool four = tile4 == nullptr || tile4[m0 / kT2M];
        if (!mbar_wait(&tmem_empty, it & 1)) fail = 1;
        fence_after();
        for (int kb = 0; kb < nkb; ++kb, ++q) {
          if (!mbar_wait(&full[st], ph)) fail = 1;
          fence_after();
          const unsigned char* sbuf = smem + (size_t)st * stage_bytes;
          const uint32_t baddr = su32(sbuf + boff);
#pragma unroll
          for (int j = 0; j < kTcKB / 32; ++j) {
            const uint64_t bdesc = smem_desc_sw64(baddr + 32 * j);
            const uint64_t ad[4] = {smem_desc_sw64(su32(sbuf) + 32 * j), smem_desc_sw64(su32(sbuf + kTcATile) + 32 * j),
                                    smem_desc_sw64(su32(sbuf + 2 * kTcATile) + 32 * j),
                                    smem_desc_sw64(su32(sbuf + 3 * kTcATile) + 32 * j)};
            if (kb == 0 && j == 0) {
              mma_i8_pair(tmem + 0 * kTcN, ad[0], bdesc, kT2Idesc, 0u);
              mma_i8_pair(tmem + 2 * kTcN, ad[2], bdesc, kT2Idesc, 0u);
              mma_i8_pair(tmem + 1 * kTcN, ad[1], bdesc, kT2Idesc, 1u);
              if (four) mma_i8_pair(tmem + 3 * kTcN, ad[3], bdesc, kT2Idesc, 1u);  // block 4 was zeroed
            } else {
#pragma unroll
              for (int a = 0; a < 3; ++a) mma_i8_pair(tmem + (uint32_t)(kTcN * a), ad[a], bdesc, kT2Idesc, 1u);
              if (four) mma_i8_pair(tmem + 3 * kTcN, ad[3], bdesc, kT2Idesc, 1u);
            }
          }
          if (q + nst < qlast) mma_commit_pair(&empty[st]);
          if (++st == nst) { st = 0; ph ^= 1u; }
        }
        mma_commit_pair(&accf);
      }
    }
  } else {
    // ---- epilogue (both CTAs): warp w reads TMEM lanes 32*(w%4).. and its
    // column half of this CTA's 128 rows
    constexpr int kOut = EPI == 2 ? kTcN / 2 : kTcN;
    constexpr int kHalf = kOut / 2;
    constexpr int kStep = EPI == 2 ? 8 : 16;
    const int quarter = warp & 3, half = warp >> 2;
    const int rl = 32 * quarter + lane;
    const uint32_t tbase = tmem + ((uint32_t)(32 * quarter) << 16);
    // block 4 of the columns this warp reads: zero before the first tile
    for (int c0 = half * kHalf; c0 < (half + 1) * kHalf; c0 += kStep) {
      tmem_st8_zero(tbase + 4 * kTcN + c0);
      tmem_st8_zero(tbase + 4 * kTcN + (EPI == 2 ? kTcN / 2 : 8) + c0);
    }
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive_cluster(tmem_empty_leader);
    for (int it = 0; it < my_tiles; ++it) {
      int m0, nt;
      tile_of(it, m0, nt);
      m0 += kTcM * (int)rank;
      const int r0 = nt * kTcN;
      const int nbase = EPI == 2 ? nt * (kTcN / 2) : r0;
      const int m = m0 + rl;
      const bool mrow = m < S;
      const RowCorr rc = row_corr(mrow ? arow[m] : 0, K);
      // the tile's weight row sums, fetched before the accumulator is ready
      uint64_t* bw = bsum[warp];
      for (int j = lane; j < kTcN; j += 32) {
        const int nn = EPI == 2 ? nbase + (j % (kTcN / 2)) : r0 + j;
        const uint64_t b = nn < N ? brow[r0 + j] : 0;
        bw[j] = b << 23;
        bw[kTcN + j] = b << 31;
      }
      __syncwarp();
      const uint64_t* bws = bw + (rc.e == 23 ? 0 : kTcN);
      if (!mbar_wait(&accf, it & 1)) fail = 1;
      fence_after();
      for (int c0 = half * kHalf; c0 < (half + 1) * kHalf; c0 += kStep) {
        uint32_t g[5][2][8];
#pragma unroll
        for (int gg = 0; gg < 5; ++gg) {
          tmem_ld8(tbase + kTcN * gg + c0, g[gg][0]);
          tmem_ld8(tbase + kTcN * gg + (EPI == 2 ? kTcN / 2 : 8) + c0, g[gg][1]);
        }
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        // these block-4 columns are read: zero them for the next tile
        tmem_st8_zero(tbase + 4 * kTcN + c0);
        tmem_st8_zero(tbase + 4 * kTcN + (EPI == 2 ? kTcN / 2 : 8) + c0);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int pr = c0 + (EPI == 2 ? (i >> 3) * (kTcN / 2) + (i & 7) : i);
          const int n = nbase + c0 + (EPI == 2 ? (i & 7) : i);
          int32_t y = 0;
          if (mrow && n < N) {
            const uint64_t acc = limb_sum(g[0][i >> 3][i & 7], g[1][i >> 3][i & 7], g[2][i >> 3][i & 7],
                                          g[3][i >> 3][i & 7], g[4][i >> 3][i & 7]) -
                                 rc.corr - bws[pr];
            y = requantize((int64_t)acc);
          }
          stage_out[rl * kTcOutStride + pr] = y;
        }
      }
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tmem_empty_leader);
      if constexpr (EPI == 1 || EPI == 2) {
        if (mrow) {
          for (int j = half * kHalf; j < (half + 1) * kHalf; ++j) {
            const int n = nbase + j;
            if (n >= N) break;
            int32_t* sp_ = &stage_out[rl * kTcOutStride + j];
            *sp_ = mul_sat(gelu_act(*sp_), EPI == 2 ? sp_[kTcN / 2] : vec[(size_t)m * ldv + n]);
          }
        }
      }
      asm volatile("bar.sync 1, %0;" ::"n"(32 * kTcEpiWarps) : "memory");  // staging complete
      for (int r = warp; r < kTcM; r += kTcEpiWarps) {
        const int mm = m0 + r;
        if (mm >= S) break;
        for (int c = lane; c < kOut; c += 32) {
          const int n = nbase + c;
          if (n < N) Y[(size_t)mm * N + n] = stage_out[r * kTcOutStride + c];
        }
      }
      asm volatile("bar.sync 1, %0;" ::"n"(32 * kTcEpiWarps) : "memory");  // staging free again
    }
  }
  fence_before();
  __syncthreads();
  cluster_sync_all();  // the leader's MMAs no longer read this CTA's shared memory
  if (fail && threadIdx.x == 0) atomicExch(&g_tc_err, 1);
  if (warp == 0) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcCols) : "memory");
  }
}

// ---------------------------------------------------------------------------
// Short row counts (a batched decode step: S <= 64 tokens).  The operands
// swap roles: the A operand is one byte plane of 128 weight rows (M = 128)
// and the B operand stacks the four activation limbs of 64 tokens (N = 256,
// B row a*64 + t).  MMA p (weight plane p) writes [P_0p | P_1p | P_2p | P_3p]
// into TMEM columns [64p, 64p + 256), so column block g = [64g, 64g + 64)
// accumulates exactly the products with shift 8g (P_g0 + P_(g-1)1): 320
// columns, each block at most two products <= 255*255*K (exact as u32 for
// K < 33025).  No MMA work is spent on padding token rows, and each stage
// moves 16 KB of weights for 128 rows instead of 12 KB for 96 rows next to
// 32 KB of mostly-padding activation limbs.
// The first K step of a tile writes every column once with accumulate off:
// plane 0 fresh over [0, 256), plane 1's limbs 0-2 onto [64, 256), plane 1's
// limb 3 fresh over [256, 320).
// EPI 0 (one K range): corrections and requantize, Y[s][n] for n < N.
// EPI 3: the raw sum of K range sp, part[sp][s][plane row], finished by
// tc_splitk_reduce_kernel (any epilogue, the gate/up pair included).
// ---------------------------------------------------------------------------
constexpr int kTsM = 128;                              // weight plane rows per tile
constexpr int kTsT = 64;                               // tokens per tile
static_assert(kTsT == kTcShortRows, "the short-row kernel covers up to kTcShortRows rows");
constexpr int kTsATile = kTsM * kTcKB;                 // 8 KB per weight plane
constexpr int kTsBTile = kTsT * kTcKB;                 // 4 KB per activation limb
constexpr int kTsStage = 2 * kTsATile + 4 * kTsBTile;  // 32 KB
constexpr int kTsStages = 6;
constexpr int kTsSmem = kTsStages * kTsStage + 1024;  // + alignment slack
constexpr uint32_t kTsIdesc = idesc_u8(4 * kTsT);      // N = 256
constexpr uint32_t kTsIdesc3 = idesc_u8(3 * kTsT);     // limbs 0-2
constexpr uint32_t kTsIdesc1 = idesc_u8(kTsT);         // limb 3

template <int EPI>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_linear_t_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap wmap,
                       const uint64_t* __restrict__ arow, const uint64_t* __restrict__ brow, int S, int N, int K,
                       int tiles_n, int ntiles, int ks, int nrows, int32_t* __restrict__ Y,
                       uint64_t* __restrict__ part) {
  extern __shared__ __align__(16) unsigned char tc_smem_raw[];
  __shared__ __align__(8) uint64_t full[kTsStages], empty[kTsStages], accf, tmem_empty;
  __shared__ uint32_t tmem_holder;
  __shared__ int fail;
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~(uintptr_t)1023);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = (K + kTcKB - 1) / kTcKB;
  const int nitems = ntiles * ks;
  const int my_tiles = blockIdx.x < nitems ? (nitems - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (threadIdx.x == 0) {
    for (int i = 0; i < kTsStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(&accf, 1);
    mbar_init(&tmem_empty, kTcEpiWarps);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fail = 0;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_holder)),
                 "r"(kTcCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = tmem_holder;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (warp == kTcEpiWarps) {
    // ---- producer: weight planes (128 rows) and activation limbs (64 tokens)
    if (lane == 0) {
      int q = 0;
      for (int it = 0; it < my_tiles; ++it) {
        const int item = blockIdx.x + it * gridDim.x, t = item / ks, sp = item % ks;
        const int r0 = (t % tiles_n) * kTsM, t0 = (t / tiles_n) * kTsT;
        const int kb0 = (int)((int64_t)nkb * sp / ks), kb1 = (int)((int64_t)nkb * (sp + 1) / ks);
        for (int kb = kb0; kb < kb1; ++kb, ++q) {
          const int st = q % kTsStages;
          if (q >= kTsStages && !mbar_wait(&empty[st], ((q / kTsStages) - 1) & 1)) fail = 1;
          unsigned char* sbuf = smem + (size_t)st * kTsStage;
          mbar_expect_tx(&full[st], kTsStage);
          tma_load_3d(sbuf, &wmap, kb * kTcKB, r0, 0, &full[st]);
          tma_load_3d(sbuf + kTsATile, &wmap, kb * kTcKB, r0, 1, &full[st]);
          for (int a = 0; a < 4; ++a)
            tma_load_3d(sbuf + 2 * kTsATile + a * kTsBTile, &amap, kb * kTcKB, t0, a, &full[st]);
        }
      }
    }
  } else if (warp == kTcEpiWarps + 1) {
    // ---- MMA issue
    if (lane == 0) {
      int q = 0, qlast = 0;
      for (int it = 0; it < my_tiles; ++it) {
        const int sp = (blockIdx.x + it * gridDim.x) % ks;
        qlast += (int)((int64_t)nkb * (sp + 1) / ks) - (int)((int64_t)nkb * sp / ks);
      }
      for (int it = 0; it < my_tiles; ++it) {
        const int sp = (blockIdx.x + it * gridDim.x) % ks;
        const int kb0 = (int)((int64_t)nkb * sp / ks), kb1 = (int)((int64_t)nkb * (sp + 1) / ks);
        if (it > 0 && !mbar_wait(&tmem_empty, (it - 1) & 1)) fail = 1;
        fence_after();
        for (int kb = kb0; kb < kb1; ++kb, ++q) {
          const int st = q % kTsStages;
          if (!mbar_wait(&full[st], (q / kTsStages) & 1)) fail = 1;
          fence_after();
          const uint32_t sb = su32(smem + (size_t)st * kTsStage);
#pragma unroll
          for (int j = 0; j < kTcKB / 32; ++j) {
            const uint64_t w0 = smem_desc_sw64(sb + 32 * j), w1 = smem_desc_sw64(sb + kTsATile + 32 * j);
            const uint64_t xb = smem_desc_sw64(sb + 2 * kTsATile + 32 * j);
            if (kb == kb0 && j == 0) {
              mma_i8(tmem, w0, xb, kTsIdesc, 0u);
              mma_i8(tmem + kTsT, w1, xb, kTsIdesc3, 1u);
              mma_i8(tmem + 4 * kTsT, w1, smem_desc_sw64(sb + 2 * kTsATile + 3 * kTsBTile + 32 * j), kTsIdesc1, 0u);
            } else {
              mma_i8(tmem, w0, xb, kTsIdesc, 1u);
              mma_i8(tmem + kTsT, w1, xb, kTsIdesc, 1u);
            }
          }
          if (q + kTsStages < qlast) mma_commit(&empty[st]);
        }
        mma_commit(&accf);
      }
    }
  } else {
    // ---- epilogue: warp w reads TMEM lanes 32*(w%4).. (weight rows) and
    // tokens [32*(w/4), 32*(w/4) + 32) of the tile
    const int quarter = warp & 3, half = warp >> 2;
    const int rl = 32 * quarter + lane;
    const uint32_t tbase = tmem + ((uint32_t)(32 * quarter) << 16);
    for (int it = 0; it < my_tiles; ++it) {
      const int item = blockIdx.x + it * gridDim.x, t = item / ks, sp = item % ks;
      const int r = (t % tiles_n) * kTsM + rl, t0 = (t / tiles_n) * kTsT;
      const bool rok = EPI == 3 ? r < nrows : r < N;
      const uint64_t bw = (EPI == 0 && rok) ? brow[r] : 0;
      if (!mbar_wait(&accf, it & 1)) fail = 1;
      fence_after();
      for (int c0 = 32 * half; c0 < 32 * half + 32; c0 += 8) {
        uint32_t g[5][8];
#pragma unroll
        for (int gg = 0; gg < 5; ++gg) tmem_ld8(tbase + kTsT * gg + c0, g[gg]);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int tok = t0 + c0 + i;
          if (rok && tok < S) {
            const uint64_t raw = limb_sum(g[0][i], g[1][i], g[2][i], g[3][i], g[4][i]);
            if (EPI == 3) part[((size_t)sp * S + tok) * nrows + r] = raw;
            else {
              const RowCorr rc = row_corr(arow[tok], K);
              Y[(size_t)tok * N + r] = requantize((int64_t)(raw - rc.corr - (bw << rc.e)));
            }
          }
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(&tmem_empty)) : "memory");
    }
  }
  fence_before();
  __syncthreads();
  if (fail && threadIdx.x == 0) atomicExch(&g_tc_err, 1);
  if (warp == 0) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcCols) : "memory");
  }
}

// Split-K finish: y = sum over splits of the raw partials, minus the row-sum
// corrections over the full K, then the epilogue.  MODE 0 plain, 1
// gelu(y) * vec[s, n] (row stride ldv), 2 gate/up pair, 3 the exact i64 sum
// before requantize (a tensor-parallel partial).
template <int MODE>
__global__ void tc_splitk_reduce_kernel(const uint64_t* __restrict__ part, int ks, int S, int nrows, int N, int K,
                                        const uint64_t* __restrict__ arow, const uint64_t* __restrict__ brow,
                                        int32_t* __restrict__ Y, int64_t* __restrict__ Y64,
                                        const int32_t* __restrict__ vec, int ldv, const TcMirrors mirror) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const size_t total = (size_t)S * N;
  for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
    const int m = (int)(e / N), n = (int)(e % N);
    const int r = MODE == 2 ? kTcN * (n / (kTcN / 2)) + n % (kTcN / 2) : n;
    const RowCorr rc = row_corr(arow[m], K);
    uint64_t acc = 0;
    for (int sp = 0; sp < ks; ++sp) acc += part[((size_t)sp * S + m) * nrows + r];
    acc -= rc.corr + (brow[r] << rc.e);
    if (MODE == 3) {
      Y64[e] = (int64_t)acc;
      for (int i = 0; i < mirror.n; ++i) mirror.p[i][e] = (int64_t)acc;  // posted stores over NVLink
      continue;
    }
    int32_t y = requantize((int64_t)acc);
    if (MODE == 2) {
      const int ru = r + kTcN / 2;
      uint64_t accu = 0;
      for (int sp = 0; sp < ks; ++sp) accu += part[((size_t)sp * S + m) * nrows + ru];
      accu -= rc.corr + (brow[ru] << rc.e);
      y = mul_sat(gelu_act(y), requantize((int64_t)accu));
    } else if (MODE == 1) {
      y = mul_sat(gelu_act(y), vec[(size_t)m * ldv + n]);
    }
    Y[e] = y;
  }
  // the mirrored sums reach the peers' memory before any later flag store
  if (MODE == 3 && mirror.n) __threadfence_system();
}

// u8 planes [planes][rows][K] -> 3D map (K, rows, planes), box (64, box_rows, 1)
bool encode_planes(void* out, const uint8_t* base, int nplanes, int rows, int K, int box_rows,
                   size_t plane_stride = 0) {
  return encode_u8_planes(out, base, nplanes, rows, K, box_rows, 1, plane_stride);
}

// launch as clusters of two CTAs (the CTA-pair kernels), with programmatic
// stream serialization
template <typename... KArgs, typename... Args>
void tc_launch_pair(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

template <typename... KArgs, typename... Args>
void tc_launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

}  // namespace

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
    else
      cudaGetLastError();
  });
  return fn;
}

bool encode_u8_planes(void* out, const uint8_t* base, int nplanes, int rows, int K, int box_rows, int box_planes,
                      size_t plane_stride) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  CUtensorMap* map = reinterpret_cast<CUtensorMap*>(out);
  const cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)rows, (cuuint64_t)nplanes};
  const cuuint64_t strides[2] = {(cuuint64_t)K,
                                 plane_stride ? (cuuint64_t)plane_stride : (cuuint64_t)rows * (cuuint64_t)K};
  const cuuint32_t box[3] = {(cuuint32_t)kTcKB, (cuuint32_t)box_rows, (cuuint32_t)box_planes};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static_assert(sizeof(CUtensorMap) <= sizeof(TcAct::map), "tensor map storage");

int tc_error_flag(bool reset) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_tc_err, sizeof(int));
  if (reset && v) {
    int z = 0;
    cudaMemcpyToSymbol(g_tc_err, &z, sizeof(int));
  }
  return v;
}

void tc_init() {
  cudaFuncSetAttribute(tc_linear_t_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTsSmem);
  cudaFuncSetAttribute(tc_linear_t_kernel<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTsSmem);
  cudaFuncSetAttribute(tc_linear_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
  cudaFuncSetAttribute(tc_linear_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
  cudaFuncSetAttribute(tc_linear_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
  cudaFuncSetAttribute(tc_linear_kernel<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
  cudaFuncSetAttribute(tc_linear2_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kT2Smem);
  cudaFuncSetAttribute(tc_linear2_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kT2Smem);
  cudaFuncSetAttribute(tc_linear2_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kT2Smem);
}

bool tc_supported() {
  static int ok = -1;
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  if (ok < 0) {
    int dev = 0, major = 0, minor = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    ok = (major == 10 && minor == 0 && encode_fn() != nullptr) ? 1 : 0;
  }
  return ok == 1;
}

bool tc_weight_eligible(const DevMat& w) {
  return w.width == 16 && w.cols > 0 && w.cols % 16 == 0 && w.cols <= kTcMaxK && w.rows > 0 &&
         (reinterpret_cast<uintptr_t>(w.p) & 15) == 0;
}

int tc_plane_rows(int rows, bool pair) { return pair ? kTcN * ((rows + kTcN / 2 - 1) / (kTcN / 2)) : rows; }

size_t tc_weight_bytes(int rows, int K, bool pair) {
  const size_t nr = (size_t)tc_plane_rows(rows, pair);
  return 2 * nr * K + nr * 8;
}

bool tc_prepare_weight(TcWeight& t, const DevMat& g, const DevMat* u, void* mem, cudaStream_t s) {
  return tc_prepare_weight_slice(t, g, u, 0, g.rows, 0, g.cols, mem, s);
}

bool tc_prepare_weight_slice(TcWeight& t, const DevMat& g, const DevMat* u, int row0, int rows, int col0, int cols,
                             void* mem, cudaStream_t s) {
  const bool pair = u != nullptr;
  t.N = rows;
  t.K = cols;
  t.pair = pair;
  t.nrows = tc_plane_rows(rows, pair);
  t.planes = static_cast<uint8_t*>(mem);
  t.rowsum = reinterpret_cast<uint64_t*>(t.planes + 2 * (size_t)t.nrows * t.K);
  tc_weight_prep_kernel<<<t.nrows, 128, 0, s>>>(static_cast<const int16_t*>(g.p),
                                                pair ? static_cast<const int16_t*>(u->p) : nullptr, rows, cols,
                                                (size_t)t.nrows * cols, t.planes, t.rowsum, row0, col0, g.cols);
  return encode_planes(t.map, t.planes, 2, t.nrows, t.K, kTcN) &&
         encode_planes(t.map_m, t.planes, 2, t.nrows, t.K, kTsM);
}

size_t tc_weight_group_bytes(const DevMat* mats, int n) {
  size_t rows = 0;
  for (int i = 0; i < n; ++i) rows += (size_t)mats[i].rows;
  return 2 * rows * mats[0].cols + rows * 8;
}

bool tc_prepare_weight_group(TcWeight* views, const DevMat* mats, int n, TcWeight& whole, void* mem,
                             cudaStream_t s) {
  const int K = mats[0].cols;
  int total = 0;
  for (int i = 0; i < n; ++i) total += mats[i].rows;
  uint8_t* base = static_cast<uint8_t*>(mem);
  uint64_t* rowsum = reinterpret_cast<uint64_t*>(base + 2 * (size_t)total * K);
  const size_t plane = (size_t)total * K;
  bool ok = true;
  int off = 0;
  for (int i = 0; i < n; ++i) {
    TcWeight& t = views[i];
    t.N = t.nrows = mats[i].rows;
    t.K = K;
    t.pair = false;
    t.planes = base + (size_t)off * K;
    t.rowsum = rowsum + off;
    tc_weight_prep_kernel<<<t.nrows, 128, 0, s>>>(static_cast<const int16_t*>(mats[i].p), nullptr, t.nrows, K, plane,
                                                  t.planes, t.rowsum, 0, 0, K);
    ok = ok && encode_planes(t.map, t.planes, 2, t.nrows, K, kTcN, plane) &&
         encode_planes(t.map_m, t.planes, 2, t.nrows, K, kTsM, plane);
    off += mats[i].rows;
  }
  whole.N = whole.nrows = total;
  whole.K = K;
  whole.pair = false;
  whole.planes = base;
  whole.rowsum = rowsum;
  return ok && encode_planes(whole.map, base, 2, total, K, kTcN) && encode_planes(whole.map_m, base, 2, total, K, kTsM);
}

size_t tc_act_bytes(int S, int K) {
  return 4 * (size_t)S * K + (size_t)S * 8 + ((size_t)(S + kT2Mrows - 1) / kT2Mrows) * 4;
}

bool tc_prepare_act(TcAct& a, const int32_t* X, int S, int K, void* mem, cudaStream_t s) {
  a.S = S;
  a.K = K;
  a.planes = static_cast<uint8_t*>(mem);
  a.rowsum = reinterpret_cast<uint64_t*>(a.planes + 4 * (size_t)S * K);
  // the tile flags are read only by the CTA-pair kernel (more than kTcM rows)
  a.tile4 = S > kTcM ? reinterpret_cast<uint32_t*>(a.rowsum + S) : nullptr;
  if (a.tile4 && cudaMemsetAsync(a.tile4, 0, ((size_t)(S + kT2Mrows - 1) / kT2Mrows) * 4, s) != cudaSuccess)
    return false;
  // few long rows (a batched decode step): more threads per row
  const int threads = (S < 2 * sm_count() && K >= 2048) ? 1024 : 256;
  tc_launch(tc_act_prep_kernel, dim3(S), dim3(threads), 0, s, X, S, K, a.planes, a.rowsum, a.tile4);
  return encode_planes(a.map, a.planes, 4, S, K, kTcM) && encode_planes(a.map_t, a.planes, 4, S, K, kTsT);
}

namespace {

// The split-K finish for partial sums part[ks][S][nrows]: corrections and
// the epilogue the output asks for.
void launch_splitk_reduce(const TcAct& a, const TcWeight& w, const TcOut& o, int ks, const uint64_t* part, int ldv,
                          cudaStream_t s) {
  const int sms = sm_count();
  const size_t total = (size_t)a.S * w.N;
  const int rblocks = (int)std::min<size_t>((total + 255) / 256, (size_t)sms * 8);
  if (o.y64)
    tc_launch(tc_splitk_reduce_kernel<3>, dim3(rblocks), dim3(256), 0, s, part, ks, a.S, w.nrows, w.N, a.K, a.rowsum,
              w.rowsum, (int32_t*)nullptr, o.y64, o.vec, ldv, o.y64_mirror);
  else if (w.pair)
    tc_launch(tc_splitk_reduce_kernel<2>, dim3(rblocks), dim3(256), 0, s, part, ks, a.S, w.nrows, w.N, a.K, a.rowsum,
              w.rowsum, o.y, (int64_t*)nullptr, o.vec, ldv, o.y64_mirror);
  else if (o.epi == kEpiGeluMul)
    tc_launch(tc_splitk_reduce_kernel<1>, dim3(rblocks), dim3(256), 0, s, part, ks, a.S, w.nrows, w.N, a.K, a.rowsum,
              w.rowsum, o.y, (int64_t*)nullptr, o.vec, ldv, o.y64_mirror);
  else
    tc_launch(tc_splitk_reduce_kernel<0>, dim3(rblocks), dim3(256), 0, s, part, ks, a.S, w.nrows, w.N, a.K, a.rowsum,
              w.rowsum, o.y, (int64_t*)nullptr, o.vec, ldv, o.y64_mirror);
}

// S <= 64: the swapped-operand kernel.  K splits are chosen by a small time
// model: a stage streams 16 KB of weights, about 0.4 us when every SM
// streams; partial sums cost 16 bytes per value and split (written, then
// read) at about 6 TB/s.  A plain output with one split needs no partials.
// Returns false (nothing launched) when partial sums are needed and the
// scratch cannot hold them.
bool launch_tc_linear_t(const TcAct& a, const TcWeight& w, const TcOut& o, int ldv, cudaStream_t s) {
  const int tiles_n = (w.nrows + kTsM - 1) / kTsM, tiles_t = (a.S + kTsT - 1) / kTsT;
  const int ntiles = tiles_n * tiles_t;
  const int nkb = (a.K + kTcKB - 1) / kTcKB;
  const int sms = sm_count();
  const bool direct_ok = !w.pair && o.epi == kEpiPlain && !o.y64;
  const size_t per_split = (size_t)a.S * w.nrows * 8;
  const double t_stage = 0.4e-6, bw = 6e12;
  int ks = 0;
  double best = 1e30;
  const int kmax = std::max(1, std::min(nkb / 2, 32));
  for (int k = 1; k <= kmax; ++k) {
    const bool partial = k > 1 || !direct_ok;
    if (partial && (!o.scratch || (size_t)k * per_split > o.scratch_bytes)) continue;
    const double waves = (double)((ntiles * k + sms - 1) / sms);
    const double t = waves * ((nkb + k - 1) / k) * t_stage + (partial ? 2.0 * k * per_split / bw : 0.0);
    if (t < best) {
      best = t;
      ks = k;
    }
  }
  if (ks == 0) return false;
  const CUtensorMap& am = *reinterpret_cast<const CUtensorMap*>(a.map_t);
  const CUtensorMap& wm = *reinterpret_cast<const CUtensorMap*>(w.map_m);
  const int grid = std::min(ntiles * ks, sms);
  if (ks == 1 && direct_ok) {
    tc_launch(tc_linear_t_kernel<0>, dim3(grid), dim3(kTcThreads), kTsSmem, s, am, wm, a.rowsum, w.rowsum, a.S, w.N,
              a.K, tiles_n, ntiles, 1, w.nrows, o.y, (uint64_t*)nullptr);
    return true;
  }
  uint64_t* part = static_cast<uint64_t*>(o.scratch);
  tc_launch(tc_linear_t_kernel<3>, dim3(grid), dim3(kTcThreads), kTsSmem, s, am, wm, a.rowsum, w.rowsum, a.S, w.N,
            a.K, tiles_n, ntiles, ks, w.nrows, (int32_t*)nullptr, part);
  launch_splitk_reduce(a, w, o, ks, part, ldv, s);
  return true;
}

}  // namespace

uint32_t* tc_act_tile4(void* mem, int S, int K) {
  return reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(mem) + 4 * (size_t)S * K + 8 * (size_t)S);
}

bool tc_attach_act(TcAct& a, int S, int K, void* mem, bool with_tile4) {
  a.S = S;
  a.K = K;
  a.planes = static_cast<uint8_t*>(mem);
  a.rowsum = reinterpret_cast<uint64_t*>(a.planes + 4 * (size_t)S * K);
  a.tile4 = with_tile4 ? tc_act_tile4(mem, S, K) : nullptr;
  return encode_planes(a.map, a.planes, 4, S, K, kTcM) && encode_planes(a.map_t, a.planes, 4, S, K, kTsT);
}

bool launch_tc_linear(const TcAct& a, const TcWeight& w, const TcOut& o, cudaStream_t s) {
  if (a.S <= kTsT && launch_tc_linear_t(a, w, o, o.ldv > 0 ? o.ldv : w.N, s)) return true;
  const int ntiles_n = (w.nrows + kTcN - 1) / kTcN;
  const int ntiles = ntiles_n * ((a.S + kTcM - 1) / kTcM);
  const int nkb = (a.K + kTcKB - 1) / kTcKB;
  const int sms = sm_count();
  const CUtensorMap& am = *reinterpret_cast<const CUtensorMap*>(a.map);
  const CUtensorMap& bm = *reinterpret_cast<const CUtensorMap*>(w.map);
  const int ldv = o.ldv > 0 ? o.ldv : w.N;
  // split K when the tiles alone would leave most SMs idle (few rows), or
  // when the caller wants the i64 sum; at least 4 stages per split
  int ks = 1;
  if (o.scratch && (ntiles * 2 <= sms || o.y64)) {
    const size_t per_split = (size_t)a.S * w.nrows * 8;
    ks = std::max(1, std::min(sms / ntiles, nkb / 4));
    ks = (int)std::min<size_t>((size_t)ks, o.scratch_bytes / per_split);
    if (ks < 1) ks = 1;
  }
  const bool split = o.scratch && (ks > 1 || o.y64) && (size_t)ks * a.S * w.nrows * 8 <= o.scratch_bytes;
  if (o.y64 && !split) return false;  // the i64 sums need the split-K scratch
  if (!split && a.S > kTcM && g_tc_pair && sms >= 2) {
    // CTA pairs: 256-token tiles, B split by plane across the pair
    const int tm = (a.S + kT2M - 1) / kT2M, tiles = tm * ntiles_n;
    const int grid = 2 * std::min(tiles, sms / 2);
    // keep the smaller operand resident in L2: all token tiles of a weight
    // tile in a row when the activation planes are the smaller
    const int m_fast = (size_t)4 * a.S * a.K < (size_t)2 * w.nrows * a.K ? 1 : 0;
    if (w.pair)
      tc_launch_pair(tc_linear2_kernel<2>, dim3(grid), dim3(kTcThreads), kT2Smem, s, am, bm, a.rowsum, w.rowsum, a.S,
                     w.N, a.K, tm, ntiles_n, m_fast, o.y, o.vec, ldv, (const uint32_t*)a.tile4);
    else if (o.epi == kEpiGeluMul)
      tc_launch_pair(tc_linear2_kernel<1>, dim3(grid), dim3(kTcThreads), kT2Smem, s, am, bm, a.rowsum, w.rowsum, a.S,
                     w.N, a.K, tm, ntiles_n, m_fast, o.y, o.vec, ldv, (const uint32_t*)a.tile4);
    else
      tc_launch_pair(tc_linear2_kernel<0>, dim3(grid), dim3(kTcThreads), kT2Smem, s, am, bm, a.rowsum, w.rowsum, a.S,
                     w.N, a.K, tm, ntiles_n, m_fast, o.y, o.vec, ldv, (const uint32_t*)a.tile4);
    return true;
  }
  if (!split) {
    const int grid = std::min(ntiles, sms);
    if (w.pair)
      tc_launch(tc_linear_kernel<2>, dim3(grid), dim3(kTcThreads), kTcSmem, s, am, bm, a.rowsum, w.rowsum, a.S, w.N,
                a.K, ntiles_n, ntiles, 1, w.nrows, o.y, o.vec, ldv, (uint64_t*)nullptr);
    else if (o.epi == kEpiGeluMul)
      tc_launch(tc_linear_kernel<1>, dim3(grid), dim3(kTcThreads), kTcSmem, s, am, bm, a.rowsum, w.rowsum, a.S, w.N,
                a.K, ntiles_n, ntiles, 1, w.nrows, o.y, o.vec, ldv, (uint64_t*)nullptr);
    else
      tc_launch(tc_linear_kernel<0>, dim3(grid), dim3(kTcThreads), kTcSmem, s, am, bm, a.rowsum, w.rowsum, a.S, w.N,
                a.K, ntiles_n, ntiles, 1, w.nrows, o.y, o.vec, ldv, (uint64_t*)nullptr);
    return true;
  }
  uint64_t* part = static_cast<uint64_t*>(o.scratch);
  const int grid = std::min(ntiles * ks, sms);
  tc_launch(tc_linear_kernel<3>, dim3(grid), dim3(kTcThreads), kTcSmem, s, am, bm, a.rowsum, w.rowsum, a.S, w.N, a.K,
            ntiles_n, ntiles, ks, w.nrows, (int32_t*)nullptr, (const int32_t*)nullptr, ldv, part);
  launch_splitk_reduce(a, w, o, ks, part, ldv, s);
  return true;
}

}  // namespace rdet
