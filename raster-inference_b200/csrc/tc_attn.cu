// Prefill attention on the 5th-generation tensor cores (tcgen05, sm_100a),
// exact: the det attention of a prompt (det_attention_prefill,
// det_kernels.rs:525-671, with the softmax of ops.rs:230-273) bit for bit.
//
// Scores.  s[i, j] = requantize(sum_k q[i, k] k[j, k]) over a head (no
// 1/sqrt(d) scale).  With q_u = q + 2^31 and k_u = k + 2^31 (u32),
//   sum q k = sum q_u k_u - 2^31 sum q_u - 2^31 sum k_u + 2^62 d   (wrapping i64)
// and q_u, k_u split into four byte limbs each, so sum q_u k_u =
// sum_{a,b} 2^(8(a+b)) P_ab with P_ab = sum_k q_a k_b, an unsigned int8
// tensor-core product.  The B operand stacks the four key limbs of a 64-key
// tile (N = 256); MMA a (query limb a) writes [P_a0 | P_a1 | P_a2 | P_a3] into
// TMEM columns [64a, 64a + 256), so column block g = [64g, 64g + 64) sums
// exactly the products of shift 8g: 7 blocks, 448 columns.  A block holds at
// most four products of at most 255^2 d each: exact as u32 for d < 16512.
//
// Softmax.  On the CUDA cores, one warp per query row: the first max comes
// from the score epilogue, then the exact exp terms, their sum, the
// ties-to-even division and the residual, exactly as the CUDA-core kernel.
// The raw weights (each in [0, 2^16]) are written as three byte planes; the
// residual that the reference adds to the first max's weight is kept per row
// and applied in the output epilogue (the add never saturates: a raw weight
// is at most 2^16 and the residual at least 2^16 - (2^31 - 1)).
//
// Weighted values.  out[i, c] = requantize(sum_j w_j v[j, c]); with
// v_u = v + 2^31, sum_j w_j v_j = sum_j raw_j v_u[j] - 2^31 sum_j raw_j +
// residual * v[first max].  Three weight limbs (A, 128 rows) times the four
// value limbs of 64 dimensions stacked as B (N = 256): 6 blocks of shift 8g,
// 384 TMEM columns, each block at most 2*255^2*n + 255*n (n keys): exact as
// u32 for n < 32961.
//
// Rows.  A tile is 128 rows: the G query heads that share a KV head times
// QB = 128 / G consecutive queries, so a tile reads each key tile once for
// all its heads.  Work items go to the persistent CTAs in descending order of
// key count, back and forth (CTA b takes items b, 2P-1-b, 2P+b, ...), which
// balances the causal triangle.  Pipelines: warp 4 loads stages with TMA (no
// multicast), warp 5 issues the MMAs, warps 0-3 drain TMEM (one thread per
// row).  Every mbarrier wait is bounded and a timeout sets the error flag.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "det_dev.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

namespace rdet {

// set when a bounded pipeline wait gives up (read by tc_attn_error_flag)
__device__ int g_ta_err = 0;

namespace {

using namespace tcx;

constexpr int kTaThreads = 192;  // warps 0-3 epilogue, 4 producer, 5 MMA
constexpr int kTaM = 128;        // rows per tile
constexpr int kTaKT = 64;        // keys per score tile / per weighted-value stage
constexpr int kQkStages = 4;
constexpr int kQkA = 4 * kTaM * 64;    // 4 query limbs x 128 rows x 64 bytes of the head dim
constexpr int kQkB = 4 * kTaKT * 64;   // 4 key limbs x 64 keys x 64 bytes
constexpr int kQkStage = kQkA + kQkB;  // 48 KB
constexpr int kQkSmem = kQkStages * kQkStage + 1024;
constexpr int kPvStages = 5;
constexpr int kPvA = 3 * kTaM * 64;    // 3 weight limbs x 128 rows x 64 keys
constexpr int kPvB = 4 * 64 * 64;      // 4 value limbs x 64 dims x 64 keys
constexpr int kPvStage = kPvA + kPvB;  // 40 KB
constexpr int kPvSmem = kPvStages * kPvStage + 1024;

constexpr uint32_t kId256 = idesc_u8(256), kId192 = idesc_u8(192), kId64 = idesc_u8(64);

struct TaParams {
  int S, Hq, Hkv, G, QB, nqt, d, nd, window, spad, cap, rows;
  const int32_t* q;   // [S, Hq, d]
  const int32_t* kc;  // [Hkv, cap, d]
  const int32_t* vc;
  int32_t* out;       // [S, Hq, d]
  uint8_t* qpl;       // [4][rows][d]
  uint64_t* qsum;     // [rows]
  uint8_t* kpl;       // [4][Hkv * spad][d]
  uint64_t* ksum;     // [Hkv * spad]
  uint8_t* vtp;       // [4][Hkv * d][spad]
  int32_t* scores;    // [rows][spad]
  uint8_t* wpl;       // [3][rows][spad]
  int32_t* rmax;      // [rows]
  int32_t* ridx;
  int32_t* resid;
  int64_t* wsum;
};

__host__ __device__ __forceinline__ int ta_win_start(const TaParams& p, int i) {
  return (p.window > 0 && i + 1 > p.window) ? i + 1 - p.window : 0;
}
// key tiles [kt0, kt1) that query tile qt reads: the keys [start(i0), last query]
__host__ __device__ __forceinline__ void ta_key_tiles(const TaParams& p, int qt, int& kt0, int& kt1) {
  const int i0 = qt * p.QB, ilast = (p.S < i0 + p.QB ? p.S : i0 + p.QB) - 1;
  kt0 = ta_win_start(p, i0) / kTaKT;
  kt1 = ilast / kTaKT + 1;
}
// the k-th item of CTA b among n items (back-and-forth rounds over the grid)
__device__ __forceinline__ int ta_item(int k, int b, int grid) { return k * grid + ((k & 1) ? grid - 1 - b : b); }

// ---------------------------------------------------------------------------
// operand planes
// ---------------------------------------------------------------------------
// Query row R of tile (kv, qt), row r = g * QB + (i - i0): four byte planes of
// q + 2^31 and their sum; rows past the prompt are zero.
__global__ void ta_prep_q_kernel(const TaParams p) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int R = blockIdx.x;
  const int item = R / kTaM, r = R % kTaM;
  const int kv = item / p.nqt, qt = item % p.nqt;
  const int g = r / p.QB, i = qt * p.QB + r % p.QB, h = kv * p.G + g;
  const size_t plane = (size_t)p.rows * p.d;
  uint32_t* dst = reinterpret_cast<uint32_t*>(p.qpl + (size_t)R * p.d);
  uint64_t sum = 0;
  for (int c = threadIdx.x; c < p.d / 4; c += blockDim.x) {
    uint32_t u[4] = {0, 0, 0, 0};
    if (i < p.S) {
      const int4 v = reinterpret_cast<const int4*>(p.q + ((size_t)i * p.Hq + h) * p.d)[c];
      u[0] = (uint32_t)v.x + 0x80000000u;
      u[1] = (uint32_t)v.y + 0x80000000u;
      u[2] = (uint32_t)v.z + 0x80000000u;
      u[3] = (uint32_t)v.w + 0x80000000u;
      sum += (uint64_t)u[0] + u[1] + u[2] + u[3];
    }
#pragma unroll
    for (int a = 0; a < 4; ++a)
      dst[a * plane / 4 + c] = ((u[0] >> (8 * a)) & 0xffu) | (((u[1] >> (8 * a)) & 0xffu) << 8) |
                               (((u[2] >> (8 * a)) & 0xffu) << 16) | (((u[3] >> (8 * a)) & 0xffu) << 24);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  __shared__ uint64_t part[8];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint64_t t = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += part[w];
    p.qsum[R] = t;
  }
}

// Key row (kv, j): four byte planes of k + 2^31 and their sum; keys past the
// prompt are zero.
__global__ void ta_prep_k_kernel(const TaParams p) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int kv = blockIdx.y, j = blockIdx.x;
  const size_t row = (size_t)kv * p.spad + j;
  const size_t plane = (size_t)p.Hkv * p.spad * p.d;
  uint32_t* dst = reinterpret_cast<uint32_t*>(p.kpl + row * p.d);
  uint64_t sum = 0;
  for (int c = threadIdx.x; c < p.d / 4; c += blockDim.x) {
    uint32_t u[4] = {0, 0, 0, 0};
    if (j < p.S) {
      const int4 v = reinterpret_cast<const int4*>(p.kc + ((size_t)kv * p.cap + j) * p.d)[c];
      u[0] = (uint32_t)v.x + 0x80000000u;
      u[1] = (uint32_t)v.y + 0x80000000u;
      u[2] = (uint32_t)v.z + 0x80000000u;
      u[3] = (uint32_t)v.w + 0x80000000u;
      sum += (uint64_t)u[0] + u[1] + u[2] + u[3];
    }
#pragma unroll
    for (int a = 0; a < 4; ++a)
      dst[a * plane / 4 + c] = ((u[0] >> (8 * a)) & 0xffu) | (((u[1] >> (8 * a)) & 0xffu) << 8) |
                               (((u[2] >> (8 * a)) & 0xffu) << 16) | (((u[3] >> (8 * a)) & 0xffu) << 24);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  __shared__ uint64_t part[8];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint64_t t = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += part[w];
    p.ksum[row] = t;
  }
}

// Values transposed for the B operand: vtp[a][kv * d + c][j] = byte a of
// v[kv][j][c] + 2^31 (zero for keys past the prompt).  One block per 64 keys
// x 64 dims of one KV head, through a shared-memory tile.
__global__ void __launch_bounds__(256) ta_prep_v_kernel(const TaParams p) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __shared__ uint32_t tile[64][65];
  const int j0 = blockIdx.x * 64, c0 = blockIdx.y * 64, kv = blockIdx.z;
  for (int e = threadIdx.x; e < 64 * 16; e += blockDim.x) {
    const int jj = e / 16, cc = 4 * (e % 16), j = j0 + jj;
    int4 v = make_int4(0, 0, 0, 0);
    uint32_t off = 0;
    if (j < p.S) {
      v = *reinterpret_cast<const int4*>(p.vc + ((size_t)kv * p.cap + j) * p.d + c0 + cc);
      off = 0x80000000u;
    }
    tile[jj][cc] = (uint32_t)v.x + off;
    tile[jj][cc + 1] = (uint32_t)v.y + off;
    tile[jj][cc + 2] = (uint32_t)v.z + off;
    tile[jj][cc + 3] = (uint32_t)v.w + off;
  }
  __syncthreads();
  const size_t plane = (size_t)p.Hkv * p.d * p.spad;
  // 4 limbs x 64 dims x 16 words of 4 keys
  for (int e = threadIdx.x; e < 4 * 64 * 16; e += blockDim.x) {
    const int a = e / (64 * 16), cc = (e / 16) % 64, jw = 4 * (e % 16);
    const uint32_t w = ((tile[jw][cc] >> (8 * a)) & 0xffu) | (((tile[jw + 1][cc] >> (8 * a)) & 0xffu) << 8) |
                       (((tile[jw + 2][cc] >> (8 * a)) & 0xffu) << 16) |
                       (((tile[jw + 3][cc] >> (8 * a)) & 0xffu) << 24);
    *reinterpret_cast<uint32_t*>(p.vtp + a * plane + ((size_t)kv * p.d + c0 + cc) * p.spad + j0 + jw) = w;
  }
}

// ---------------------------------------------------------------------------
// scores: QK^T on the tensor cores, requantized, with each row's first max
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kTaThreads, 1)
    ta_qk_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap, const TaParams p) {
  extern __shared__ __align__(16) unsigned char ta_smem_raw[];
  __shared__ __align__(8) uint64_t full[kQkStages], empty[kQkStages], accf, tmem_empty;
  __shared__ uint32_t tmem_holder;
  __shared__ int fail;
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(ta_smem_raw) + 1023) & ~(uintptr_t)1023);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nitems = p.Hkv * p.nqt, grid = gridDim.x, b = blockIdx.x;
  const int nrounds = (nitems + grid - 1) / grid;
  const int ns = p.d / 64;  // stages per key tile
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (threadIdx.x == 0) {
    for (int i = 0; i < kQkStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(&accf, 1);
    mbar_init(&tmem_empty, 4);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fail = 0;
  }
  if (warp == 0) tmem_alloc512(&tmem_holder);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = tmem_holder;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (warp == 4) {
    if (lane == 0) {
      int q = 0;
      for (int k = 0; k < nrounds; ++k) {
        const int e = ta_item(k, b, grid);
        if (e >= nitems) continue;
        const int qt = p.nqt - 1 - e / p.Hkv, kv = e % p.Hkv;
        int kt0, kt1;
        ta_key_tiles(p, qt, kt0, kt1);
        const int row0 = (kv * p.nqt + qt) * kTaM;
        for (int kt = kt0; kt < kt1; ++kt)
          for (int s = 0; s < ns; ++s, ++q) {
            const int st = q % kQkStages;
            if (q >= kQkStages && !mbar_wait(&empty[st], ((q / kQkStages) - 1) & 1)) fail = 1;
            unsigned char* buf = smem + (size_t)st * kQkStage;
            mbar_expect_tx(&full[st], kQkStage);
            tma_load_3d(buf, &qmap, 64 * s, row0, 0, &full[st]);
            tma_load_3d(buf + kQkA, &kmap, 64 * s, kv * p.spad + kt * kTaKT, 0, &full[st]);
          }
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {
      int qtotal = 0;
      for (int k = 0; k < nrounds; ++k) {
        const int e = ta_item(k, b, grid);
        if (e >= nitems) continue;
        int kt0, kt1;
        ta_key_tiles(p, p.nqt - 1 - e / p.Hkv, kt0, kt1);
        qtotal += (kt1 - kt0) * ns;
      }
      int q = 0, tc = 0;
      for (int k = 0; k < nrounds; ++k) {
        const int e = ta_item(k, b, grid);
        if (e >= nitems) continue;
        int kt0, kt1;
        ta_key_tiles(p, p.nqt - 1 - e / p.Hkv, kt0, kt1);
        for (int kt = kt0; kt < kt1; ++kt, ++tc) {
          if (tc > 0 && !mbar_wait(&tmem_empty, (tc - 1) & 1)) fail = 1;
          fence_after();
          for (int s = 0; s < ns; ++s, ++q) {
            const int st = q % kQkStages;
            if (!mbar_wait(&full[st], (q / kQkStages) & 1)) fail = 1;
            fence_after();
            const uint32_t base = su32(smem + (size_t)st * kQkStage);
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const uint64_t a0 = smem_desc_sw64(base + 32 * j), a1 = smem_desc_sw64(base + 8192 + 32 * j),
                             a2 = smem_desc_sw64(base + 16384 + 32 * j), a3 = smem_desc_sw64(base + 24576 + 32 * j);
              const uint64_t bd = smem_desc_sw64(base + kQkA + 32 * j);
              if (s == 0 && j == 0) {
                // every column written once with accumulate off first
                const uint64_t b3 = smem_desc_sw64(base + kQkA + 3 * 4096);
                mma_i8(tmem + 0, a0, bd, kId256, 0u);
                mma_i8(tmem + 64, a1, bd, kId192, 1u);
                mma_i8(tmem + 256, a1, b3, kId64, 0u);
                mma_i8(tmem + 128, a2, bd, kId192, 1u);
                mma_i8(tmem + 320, a2, b3, kId64, 0u);
                mma_i8(tmem + 192, a3, bd, kId192, 1u);
                mma_i8(tmem + 384, a3, b3, kId64, 0u);
              } else {
                mma_i8(tmem + 0, a0, bd, kId256, 1u);
                mma_i8(tmem + 64, a1, bd, kId256, 1u);
                mma_i8(tmem + 128, a2, bd, kId256, 1u);
                mma_i8(tmem + 192, a3, bd, kId256, 1u);
              }
            }
            if (q + kQkStages < qtotal) mma_commit(&empty[st]);
          }
          mma_commit(&accf);
        }
      }
    }
  } else {
    // ---- epilogue: thread r drains TMEM lane r (tile row r)
    const int r = 32 * warp + lane;
    const uint32_t tbase = tmem + ((uint32_t)(32 * warp) << 16);
    const uint64_t dcorr = (uint64_t)p.d << 62;
    int tc = 0;
    for (int k = 0; k < nrounds; ++k) {
      const int e = ta_item(k, b, grid);
      if (e >= nitems) continue;
      const int qt = p.nqt - 1 - e / p.Hkv, kv = e % p.Hkv;
      int kt0, kt1;
      ta_key_tiles(p, qt, kt0, kt1);
      const int R = (kv * p.nqt + qt) * kTaM + r;
      const int i = qt * p.QB + r % p.QB;
      const bool rowok = i < p.S;
      const int st_i = ta_win_start(p, i);
      const uint64_t qs = p.qsum[R];
      int32_t best = INT32_MIN, bidx = INT32_MAX;
      for (int kt = kt0; kt < kt1; ++kt, ++tc) {
        if (!mbar_wait(&accf, tc & 1)) fail = 1;
        fence_after();
        const uint64_t* ks = p.ksum + (size_t)kv * p.spad + kt * kTaKT;
        int32_t* srow = p.scores + (size_t)R * p.spad + kt * kTaKT;
        for (int c0 = 0; c0 < kTaKT; c0 += 8) {
          uint32_t gq[7][8];
#pragma unroll
          for (int gg = 0; gg < 7; ++gg) tmem_ld8(tbase + 64 * gg + c0, gq[gg]);
          tmem_wait_ld();
          int32_t v[8];
#pragma unroll
          for (int x = 0; x < 8; ++x) {
            uint64_t acc = (uint64_t)gq[0][x] + ((uint64_t)gq[1][x] << 8) + ((uint64_t)gq[2][x] << 16) +
                           ((uint64_t)gq[3][x] << 24) + ((uint64_t)gq[4][x] << 32) + ((uint64_t)gq[5][x] << 40) +
                           ((uint64_t)gq[6][x] << 48);
            acc = acc - ((qs + ks[c0 + x]) << 31) + dcorr;
            v[x] = requantize((int64_t)acc);
            const int j = kt * kTaKT + c0 + x;
            if (rowok && j >= st_i && j <= i && (v[x] > best || bidx == INT32_MAX)) {
              best = v[x];
              bidx = j;
            }
          }
          reinterpret_cast<int4*>(srow + c0)[0] = make_int4(v[0], v[1], v[2], v[3]);
          reinterpret_cast<int4*>(srow + c0)[1] = make_int4(v[4], v[5], v[6], v[7]);
        }
        fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tmem_empty);
      }
      if (rowok) {
        p.rmax[R] = best;
        p.ridx[R] = bidx;
      }
    }
  }
  fence_before();
  __syncthreads();
  if (fail && threadIdx.x == 0) atomicExch(&g_ta_err, 1);
  if (warp == 0) {
    fence_after();
    tmem_dealloc512(tmem);
  }
}

// ---------------------------------------------------------------------------
// exact softmax per row (CUDA cores): raw weights as three byte planes over
// the key tiles the weighted-value pass reads, their exact sum, the residual
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) ta_softmax_kernel(const TaParams p) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int R = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (R >= p.rows) return;
  const int item = R / kTaM, r = R % kTaM;
  const int qt = item % p.nqt;
  const int i = qt * p.QB + r % p.QB;
  int kt0, kt1;
  ta_key_tiles(p, qt, kt0, kt1);
  const size_t plane = (size_t)p.rows * p.spad;
  uint8_t* w0 = p.wpl + (size_t)R * p.spad;
  const int jlo = kt0 * kTaKT, jhi = kt1 * kTaKT;
  if (i >= p.S) {
    for (int j = jlo + 4 * lane; j < jhi; j += 128) {
      *reinterpret_cast<uint32_t*>(w0 + j) = 0;
      *reinterpret_cast<uint32_t*>(w0 + plane + j) = 0;
      *reinterpret_cast<uint32_t*>(w0 + 2 * plane + j) = 0;
    }
    return;
  }
  const int st = ta_win_start(p, i);
  const int32_t mx = p.rmax[R];
  const int32_t* sc = p.scores + (size_t)R * p.spad;
  uint64_t sum = 0;
  for (int j = (st & ~3) + 4 * lane; j <= i; j += 128) {
    const int4 v = *reinterpret_cast<const int4*>(sc + j);
    const int32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int x = 0; x < 4; ++x)
      if (j + x >= st && j + x <= i) sum += (uint64_t)exp_term(vv[x], mx);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  int64_t wsum = 0;
  for (int j = jlo + 4 * lane; j < jhi; j += 128) {
    uint32_t b0 = 0, b1 = 0, b2 = 0;
    if (j + 3 >= st && j <= i) {
      const int4 v = *reinterpret_cast<const int4*>(sc + j);
      const int32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int x = 0; x < 4; ++x) {
        if (j + x >= st && j + x <= i) {
          const uint32_t w = (uint32_t)softmax_weight(exp_term(vv[x], mx), (int64_t)sum);
          wsum += w;
          b0 |= (w & 0xffu) << (8 * x);
          b1 |= ((w >> 8) & 0xffu) << (8 * x);
          b2 |= (w >> 16) << (8 * x);
        }
      }
    }
    *reinterpret_cast<uint32_t*>(w0 + j) = b0;
    *reinterpret_cast<uint32_t*>(w0 + plane + j) = b1;
    *reinterpret_cast<uint32_t*>(w0 + 2 * plane + j) = b2;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, o);
  if (lane == 0) {
    p.wsum[R] = wsum;
    p.resid[R] = sub_sat(kOneAct, wsum > INT32_MAX ? INT32_MAX : (int32_t)wsum);
  }
}

// ---------------------------------------------------------------------------
// weighted values: W V on the tensor cores, 64 output dims per item
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kTaThreads, 1)
    ta_pv_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap vmap, const TaParams p) {
  extern __shared__ __align__(16) unsigned char ta_smem_raw[];
  __shared__ __align__(8) uint64_t full[kPvStages], empty[kPvStages], accf, tmem_empty;
  __shared__ uint32_t tmem_holder;
  __shared__ int fail;
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(ta_smem_raw) + 1023) & ~(uintptr_t)1023);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per_qt = p.Hkv * p.nd;
  const int nitems = p.nqt * per_qt, grid = gridDim.x, b = blockIdx.x;
  const int nrounds = (nitems + grid - 1) / grid;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (threadIdx.x == 0) {
    for (int i = 0; i < kPvStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(&accf, 1);
    mbar_init(&tmem_empty, 4);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fail = 0;
  }
  if (warp == 0) tmem_alloc512(&tmem_holder);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = tmem_holder;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (warp == 4) {
    if (lane == 0) {
      int q = 0;
      for (int k = 0; k < nrounds; ++k) {
        const int e = ta_item(k, b, grid);
        if (e >= nitems) continue;
        const int qt = p.nqt - 1 - e / per_qt, kv = (e % per_qt) / p.nd, dc = e % p.nd;
        int kt0, kt1;
        ta_key_tiles(p, qt, kt0, kt1);
        const int row0 = (kv * p.nqt + qt) * kTaM;
        for (int kt = kt0; kt < kt1; ++kt, ++q) {
          const int st = q % kPvStages;
          if (q >= kPvStages && !mbar_wait(&empty[st], ((q / kPvStages) - 1) & 1)) fail = 1;
          unsigned char* buf = smem + (size_t)st * kPvStage;
          mbar_expect_tx(&full[st], kPvStage);
          tma_load_3d(buf, &wmap, kt * kTaKT, row0, 0, &full[st]);
          tma_load_3d(buf + kPvA, &vmap, kt * kTaKT, kv * p.d + dc * 64, 0, &full[st]);
        }
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {
      int qtotal = 0;
      for (int k = 0; k < nrounds; ++k) {
        const int e = ta_item(k, b, grid);
        if (e >= nitems) continue;
        int kt0, kt1;
        ta_key_tiles(p, p.nqt - 1 - e / per_qt, kt0, kt1);
        qtotal += kt1 - kt0;
      }
      int q = 0, tc = 0;
      for (int k = 0; k < nrounds; ++k) {
        const int e = ta_item(k, b, grid);
        if (e >= nitems) continue;
        int kt0, kt1;
        ta_key_tiles(p, p.nqt - 1 - e / per_qt, kt0, kt1);
        if (tc > 0 && !mbar_wait(&tmem_empty, (tc - 1) & 1)) fail = 1;
        fence_after();
        for (int kt = kt0; kt < kt1; ++kt, ++q) {
          const int st = q % kPvStages;
          if (!mbar_wait(&full[st], (q / kPvStages) & 1)) fail = 1;
          fence_after();
          const uint32_t base = su32(smem + (size_t)st * kPvStage);
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const uint64_t a0 = smem_desc_sw64(base + 32 * j), a1 = smem_desc_sw64(base + 8192 + 32 * j),
                           a2 = smem_desc_sw64(base + 16384 + 32 * j);
            const uint64_t bd = smem_desc_sw64(base + kPvA + 32 * j);
            if (kt == kt0 && j == 0) {
              const uint64_t b3 = smem_desc_sw64(base + kPvA + 3 * 4096);
              mma_i8(tmem + 0, a0, bd, kId256, 0u);
              mma_i8(tmem + 64, a1, bd, kId192, 1u);
              mma_i8(tmem + 256, a1, b3, kId64, 0u);
              mma_i8(tmem + 128, a2, bd, kId192, 1u);
              mma_i8(tmem + 320, a2, b3, kId64, 0u);
            } else {
              mma_i8(tmem + 0, a0, bd, kId256, 1u);
              mma_i8(tmem + 64, a1, bd, kId256, 1u);
              mma_i8(tmem + 128, a2, bd, kId256, 1u);
            }
          }
          if (q + kPvStages < qtotal) mma_commit(&empty[st]);
        }
        mma_commit(&accf);
        ++tc;
      }
    }
  } else {
    const int r = 32 * warp + lane;
    const uint32_t tbase = tmem + ((uint32_t)(32 * warp) << 16);
    int tc = 0;
    for (int k = 0; k < nrounds; ++k) {
      const int e = ta_item(k, b, grid);
      if (e >= nitems) continue;
      const int qt = p.nqt - 1 - e / per_qt, kv = (e % per_qt) / p.nd, dc = e % p.nd;
      const int R = (kv * p.nqt + qt) * kTaM + r;
      const int g = r / p.QB, i = qt * p.QB + r % p.QB;
      const bool rowok = i < p.S;
      uint64_t wcorr = 0;
      int32_t res = 0;
      const int32_t* vrow = nullptr;
      if (rowok) {
        wcorr = (uint64_t)p.wsum[R] << 31;
        res = p.resid[R];
        vrow = p.vc + ((size_t)kv * p.cap + p.ridx[R]) * p.d + dc * 64;
      }
      if (!mbar_wait(&accf, tc & 1)) fail = 1;
      fence_after();
      int32_t* orow = p.out + ((size_t)i * p.Hq + kv * p.G + g) * p.d + dc * 64;
      for (int c0 = 0; c0 < 64; c0 += 8) {
        uint32_t gq[6][8];
#pragma unroll
        for (int gg = 0; gg < 6; ++gg) tmem_ld8(tbase + 64 * gg + c0, gq[gg]);
        tmem_wait_ld();
        if (rowok) {
          int32_t y[8];
#pragma unroll
          for (int x = 0; x < 8; ++x) {
            uint64_t acc = (uint64_t)gq[0][x] + ((uint64_t)gq[1][x] << 8) + ((uint64_t)gq[2][x] << 16) +
                           ((uint64_t)gq[3][x] << 24) + ((uint64_t)gq[4][x] << 32) + ((uint64_t)gq[5][x] << 40);
            acc = acc - wcorr + (uint64_t)((int64_t)res * vrow[c0 + x]);
            y[x] = requantize((int64_t)acc);
          }
          reinterpret_cast<int4*>(orow + c0)[0] = make_int4(y[0], y[1], y[2], y[3]);
          reinterpret_cast<int4*>(orow + c0)[1] = make_int4(y[4], y[5], y[6], y[7]);
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tmem_empty);
      ++tc;
    }
  }
  fence_before();
  __syncthreads();
  if (fail && threadIdx.x == 0) atomicExch(&g_ta_err, 1);
  if (warp == 0) {
    fence_after();
    tmem_dealloc512(tmem);
  }
}

template <typename... KArgs, typename... Args>
void ta_launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
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

size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

// workspace layout for (S, Hq, Hkv, d); returns total bytes and fills p's
// pointers when base is not null
size_t ta_layout(TaParams& p, unsigned char* base) {
  size_t off = 0;
  auto take = [&](size_t bytes) {
    unsigned char* at = base ? base + off : nullptr;
    off += align256(bytes);
    return at;
  };
  const size_t rows = (size_t)p.rows, spad = (size_t)p.spad, d = (size_t)p.d;
  p.qpl = take(4 * rows * d);
  p.qsum = reinterpret_cast<uint64_t*>(take(rows * 8));
  p.kpl = take(4 * (size_t)p.Hkv * spad * d);
  p.ksum = reinterpret_cast<uint64_t*>(take((size_t)p.Hkv * spad * 8));
  p.vtp = take(4 * (size_t)p.Hkv * d * spad);
  p.scores = reinterpret_cast<int32_t*>(take(rows * spad * 4));
  p.wpl = take(3 * rows * spad);
  p.rmax = reinterpret_cast<int32_t*>(take(rows * 4));
  p.ridx = reinterpret_cast<int32_t*>(take(rows * 4));
  p.resid = reinterpret_cast<int32_t*>(take(rows * 4));
  p.wsum = reinterpret_cast<int64_t*>(take(rows * 8));
  return off;
}

bool ta_shape(TaParams& p, int S, int Hq, int Hkv, int d) {
  if (S < 1 || Hkv < 1 || Hq % Hkv != 0 || d < 64 || d % 64 != 0 || d > 16384 || S > 32768) return false;
  const int G = Hq / Hkv;
  if (G > kTaM || kTaM % G != 0) return false;
  p.S = S;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.G = G;
  p.QB = kTaM / G;
  p.nqt = (S + p.QB - 1) / p.QB;
  p.d = d;
  p.nd = d / 64;
  p.spad = (S + kTaKT - 1) / kTaKT * kTaKT;
  p.rows = Hkv * p.nqt * kTaM;
  return true;
}

}  // namespace

int tc_attn_error_flag(bool reset) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_ta_err, sizeof(int));
  if (reset && v) {
    int z = 0;
    cudaMemcpyToSymbol(g_ta_err, &z, sizeof(int));
  }
  return v;
}

void tc_attn_init() {
  cudaFuncSetAttribute(ta_qk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kQkSmem);
  cudaFuncSetAttribute(ta_pv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPvSmem);
}

size_t tc_attn_ws_bytes(int S, int Hq, int Hkv, int d) {
  TaParams p{};
  if (!ta_shape(p, S, Hq, Hkv, d)) return 0;
  return ta_layout(p, nullptr);
}

bool tc_attn_eligible(int S, int Hq, int Hkv, int d) {
  TaParams p{};
  return tc_supported() && ta_shape(p, S, Hq, Hkv, d);
}

bool launch_attn_prefill_tc(const AttnPrefillArgs& a, void* ws, size_t ws_bytes, cudaStream_t s) {
  TaParams p{};
  if (!tc_supported() || !ta_shape(p, a.S, a.Hq, a.Hkv, a.d) || a.cap < a.S) return false;
  if (((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k_cache) |
        reinterpret_cast<uintptr_t>(a.v_cache) | reinterpret_cast<uintptr_t>(a.out)) & 15) != 0)
    return false;
  p.window = a.window;
  p.cap = a.cap;
  p.q = a.q;
  p.kc = a.k_cache;
  p.vc = a.v_cache;
  p.out = a.out;
  if (ta_layout(p, nullptr) > ws_bytes || !ws) return false;
  ta_layout(p, static_cast<unsigned char*>(ws));
  alignas(64) CUtensorMap qmap, kmap, wmap, vmap;
  if (!encode_u8_planes(&qmap, p.qpl, 4, p.rows, p.d, kTaM, 4, 0) ||
      !encode_u8_planes(&kmap, p.kpl, 4, p.Hkv * p.spad, p.d, kTaKT, 4, 0) ||
      !encode_u8_planes(&wmap, p.wpl, 3, p.rows, p.spad, kTaM, 3, 0) ||
      !encode_u8_planes(&vmap, p.vtp, 4, p.Hkv * p.d, p.spad, 64, 4, 0))
    return false;
  const int sms = sm_count();
  ta_launch(ta_prep_q_kernel, dim3(p.rows), dim3(128), 0, s, p);
  ta_launch(ta_prep_k_kernel, dim3(p.spad, p.Hkv), dim3(128), 0, s, p);
  ta_launch(ta_prep_v_kernel, dim3(p.spad / 64, p.nd, p.Hkv), dim3(256), 0, s, p);
  ta_launch(ta_qk_kernel, dim3(std::min(sms, p.Hkv * p.nqt)), dim3(kTaThreads), (size_t)kQkSmem, s, qmap, kmap, p);
  ta_launch(ta_softmax_kernel, dim3((p.rows + 7) / 8), dim3(256), 0, s, p);
  ta_launch(ta_pv_kernel, dim3(std::min(sms, p.Hkv * p.nqt * p.nd)), dim3(kTaThreads), (size_t)kPvSmem, s, wmap,
            vmap, p);
  return true;
}

}  // namespace rdet
