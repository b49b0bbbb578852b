// Batched decode attention on the 5th-generation tensor cores (tcgen05,
// sm_100a), exact: attention_output_into (det_kernels.rs:340-367, with the
// softmax of ops.rs:230-273) for every sequence of a batched decode step, bit
// for bit the same as the CUDA-core cluster kernel.
//
// One thread-block cluster per (sequence, group of GC query heads sharing a
// KV head); CTA r of the cluster takes keys [n r / CL, n (r+1) / CL) of the
// sequence's window.  The KV cache keeps its i32 row layout: tiled TMA
// loads (a 2D tensor map per sequence and cache, 128-byte swizzle) bring raw
// cache tiles into a shared-memory ring, and the CTA converts them there into
// unsigned byte-limb planes (the 64-byte swizzle layout the MMA descriptors
// read), so nothing else in the library changes.
//
// Scores.  With k_u = k + 2^31 and q_u = q + 2^31 (u32),
//   sum k q = sum k_u q_u - 2^31 sum q_u - 2^31 sum k_u + 2^62 d  (wrapping i64)
// and sum k_u q_u = sum_{a,b} 2^(8(a+b)) P_b[a], P_b[a] = sum_dim kbyte_b
// qbyte_a.  The keys are the MMA's M = 128 rows (A = key limb plane b); the
// B operand stacks the four query limbs of each of the GC heads (row 4h + a)
// and one row of ones (row 16, N = 32), so one MMA per key limb writes P_b
// for all heads and the key's limb-b byte sum, from which sum k_u follows:
// 128 TMEM columns per 128-key tile, double-buffered.  Each entry is at most
// 255^2 d: exact in the s32 accumulator for d <= 512.
//
// Softmax.  First max, exp terms, their sum, the ties-to-even division and
// the residual on the CUDA cores, cluster-wide through distributed shared
// memory, exactly as the cluster kernel.
//
// Weighted values.  With v_u = v + 2^31, sum_j w_j v_j = sum_j w_j v_u[j] -
// 2^31 sum_j w_j; a weight is at most 2^16, three byte limbs.  Value tiles
// are converted transposed (A = value limb plane b: 128 dims x 64 keys), the
// B operand holds the weight limbs (row 4h + a), one MMA per value limb and
// 32 keys; per 128 dims 64 TMEM columns accumulate over the CTA's keys, each
// entry at most 255^2 n for n keys: exact for n <= 33000.
//
// Warp roles, coupled only by mbarriers: warp 8 issues the TMA loads into a
// ring of three 32 KB slots (score tiles, then value tiles, so the first
// value tiles load while the softmax runs), warps 0-7 convert each slot into
// one of two plane buffers, warp 9 issues the MMAs of a plane buffer once all
// converters have written it, and warps 10-13 drain the double-buffered score
// accumulators as tiles complete.  The softmax and the cluster combine use
// every warp.  Every mbarrier wait is bounded: a wait that gives up sets the
// library's pipeline error flag (the host raises an error).  No load uses
// cluster multicast.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cooperative_groups.h>
#include <cstdint>
#include <cstdlib>
#include <mutex>
#include <vector>

#include "det_dev.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

namespace rdet {

// set when a bounded wait gives up (read by tc_attn_dec_error_flag)
__device__ int g_tad_err = 0;

namespace {

namespace cg = cooperative_groups;

// warps 0-7 convert raw tiles to limb planes, warp 8 issues the TMA loads,
// warp 9 the MMAs, warps 10-13 drain the score accumulators; all of them
// share the softmax and combine phases
constexpr int kTdThreads = 448;
constexpr int kTdWarps = kTdThreads / 32;
constexpr int kTdConv = 256;  // converter threads
constexpr int kTdProdWarp = 8, kTdMmaWarp = 9, kTdEpiWarp = 10;
constexpr int kTdKeys = 128;                 // keys per score tile (MMA M)
constexpr int kTdVKeys = 64;                 // keys per value tile
constexpr int kTdBox = 64 * 128;             // one TMA box: 64 cache rows x 32 i32, 128-byte swizzle
constexpr int kTdSlot = 4 * kTdBox;           // 32 KB: 128 keys x 64 dims, or 64 keys x 128 dims
constexpr int kTdSlots = 3;
constexpr int kTdPlane = 128 * 64;           // one limb plane tile [128][64 B]
constexpr int kTdPlanes = 4 * kTdPlane;      // 32 KB
constexpr int kTdMaxRows = 1280;             // keys per CTA at most
constexpr uint32_t kTdId16 = tcx::idesc_u8(16), kTdId32 = tcx::idesc_u8(32);

struct TdLayout {  // byte offsets in the 1024-aligned dynamic shared memory
  int ring, planes, qpl, wpl, sc, total;
};
__host__ __device__ inline TdLayout td_layout(int d, int rmax, int gc) {
  TdLayout L;
  int o = 0;
  L.ring = o; o += kTdSlots * kTdSlot;
  o = (o + 1023) & ~1023;
  L.planes = o; o += 2 * kTdPlanes;
  L.qpl = o; o += (d / 64) * 2048;
  L.wpl = o; o += ((rmax + 63) / 64) * 1024;
  L.sc = o; o += gc * rmax * 4;
  L.total = o + 1024;  // alignment slack
  return L;
}

__device__ __forceinline__ uint32_t td_su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void td_fence_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void td_cp4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(td_su32(dst)), "l"(src) : "memory");
}
// tiled 2D TMA load of one box (the tensor map lives in global memory)
__device__ __forceinline__ void td_tma2d(void* dst, const void* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(td_su32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(td_su32(bar))
      : "memory");
}
// byte offset of (row r, 16-byte chunk c) in a [rows][128 B] box in the
// 128-byte swizzle (16-byte chunk index XOR the row's low three bits)
__device__ __forceinline__ int sw128(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld1(uint32_t taddr, uint32_t& r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr));
}

// byte offset of (row r, 16-byte chunk c) in a [rows][64 B] tile in the
// 64-byte swizzle (16-byte chunk index XOR bits 1-2 of the row)
__device__ __forceinline__ int sw64(int r, int c) { return r * 64 + ((c ^ ((r >> 1) & 3)) << 4); }

// 4 x 4 byte transpose: out[b] = byte b of w0..w3 (w0 in the low byte)
__device__ __forceinline__ void bytes_t4(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3, uint32_t (&o)[4]) {
  const uint32_t t0 = __byte_perm(w0, w1, 0x5140), t1 = __byte_perm(w2, w3, 0x5140);
  const uint32_t t2 = __byte_perm(w0, w1, 0x7362), t3 = __byte_perm(w2, w3, 0x7362);
  o[0] = __byte_perm(t0, t1, 0x5410);
  o[1] = __byte_perm(t0, t1, 0x7632);
  o[2] = __byte_perm(t2, t3, 0x5410);
  o[3] = __byte_perm(t2, t3, 0x7632) ^ 0x80808080u;  // byte 3 of x + 2^31
}

__device__ __forceinline__ void td_first_max_merge(int32_t& v, int32_t& ix, int32_t ov, int32_t oi) {
  if (oi != INT32_MAX && (ix == INT32_MAX || ov > v || (ov == v && oi < ix))) { v = ov; ix = oi; }
}
__device__ __forceinline__ int64_t td_warp_sum(int64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

struct TdArgs {
  AttnDecodeArgs a;
  int rmax;
};

template <int GC>
__global__ void __launch_bounds__(kTdThreads, 1) attn_dec_tc_kernel(const TdArgs ta) {
  const AttnDecodeArgs& a = ta.a;
  const int rmax = ta.rmax;
  extern __shared__ __align__(16) unsigned char td_smem_raw[];
  unsigned char* sm =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(td_smem_raw) + 1023) & ~(uintptr_t)1023);
  cg::cluster_group cl = cg::this_cluster();
  const int CL = (int)cl.num_blocks(), rank = (int)cl.block_rank();
  const int d = a.d, ns = d / 64, nd = d / 128;
  const int G = a.group ? a.group : a.Hq / a.Hkv;
  const int qh0 = blockIdx.y * GC;
  const int kvh = (a.head0 + qh0) / G;
  const TdLayout Ly = td_layout(d, rmax, GC);
  unsigned char* ring = sm + Ly.ring;
  unsigned char* planes = sm + Ly.planes;
  unsigned char* qpl = sm + Ly.qpl;
  unsigned char* wpl = sm + Ly.wpl;
  int32_t* sc = reinterpret_cast<int32_t*>(sm + Ly.sc);       // [GC][rmax] scores, then weights
  int64_t* ex = reinterpret_cast<int64_t*>(planes);           // [GC][rmax] exp terms (between the MMA phases)
  int64_t* pacc = reinterpret_cast<int64_t*>(ring);           // [GC][d] partial weighted sums (after the last tile)
  // planes_full[p]: every thread converted its part of plane buffer p;
  // mma_done[p]: the MMAs reading plane buffer p completed
  // full[s] / empty[s]: ring slot s loaded (TMA bytes) / converted by every thread
  __shared__ __align__(8) uint64_t full[kTdSlots], empty[kTdSlots], planes_full[2], mma_done[2], acc_full[2],
      acc_empty[2], pv_full;
  __shared__ uint32_t tmem_holder;
  __shared__ uint64_t qsum[4];
  __shared__ int32_t s_max[GC], s_idx[GC], g_max[GC], g_idx[GC], g_res[GC];
  __shared__ int64_t s_sum[GC], s_wsum[GC], g_sum[GC];
  __shared__ int32_t wm[kTdWarps][GC], wi[kTdWarps][GC];
  __shared__ int64_t ws[kTdWarps][GC];
  __shared__ int32_t vmx[GC][256];
  __shared__ int s_fail;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (tid == 0) {
    for (int i = 0; i < kTdSlots; ++i) {
      tcx::mbar_init(&full[i], 1);
      tcx::mbar_init(&empty[i], kTdConv);
    }
    for (int i = 0; i < 2; ++i) {
      tcx::mbar_init(&planes_full[i], kTdConv);
      tcx::mbar_init(&mma_done[i], 1);
      tcx::mbar_init(&acc_full[i], 1);
      tcx::mbar_init(&acc_empty[i], 128);
    }
    tcx::mbar_init(&pv_full, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_fail = 0;
  }
  if (warp == 0) tcx::tmem_alloc512(&tmem_holder);
  tcx::fence_before();
  __syncthreads();
  tcx::fence_after();
  const uint32_t tmem = tmem_holder;
  asm volatile("griddepcontrol.wait;" ::: "memory");

  const int brow = a.row_order ? a.row_order[blockIdx.z] : (int)blockIdx.z;
  const int32_t* const vc = a.vc_rows[brow];
  const int capr = a.cap_rows[brow];
  const int32_t* const qrow = a.q + (size_t)brow * a.Hq * d;
  int32_t* const orow = a.out + (size_t)brow * a.Hq * d;
  const int len = *a.pos_rows[brow] + 1;
  const int start = (a.window > 0 && len > a.window) ? len - a.window : 0;
  const int n = len - start;
  const int lo = (int)((int64_t)n * rank / CL), hi = (int)((int64_t)n * (rank + 1) / CL);
  const int rows = hi - lo;
  const int ntile = (rows + kTdKeys - 1) / kTdKeys;
  const int nq = ntile * ns;                                  // score stages
  const int nkb = (rows + kTdVKeys - 1) / kTdVKeys;
  const int total = nq + nkb * nd;                            // + value stages
  // a converter thread's row (key or dim) and half of the columns (dims or keys)
  const int crow = tid & 127, half = (tid >> 7) & 1;

  auto wait = [&](uint64_t* bar, uint32_t parity) {
    if (!tcx::mbar_wait(bar, parity)) s_fail = 1;
  };
  // Stage u -> slot u % kTdSlots by the producer: four TMA boxes (score stage:
  // keys [128 t, +128) x dims [64 s, +64); value stage: keys [64 kb, +64) x
  // dims [128 db, +128)), rows past the cache read as zero, rows past this
  // CTA's keys are ignored.  Issued once every converter thread has
  // converted the slot's previous stage.
  const unsigned char* const maps = a.map_rows[brow] + (size_t)a.map_layer * 256;
  const int y0 = kvh * capr + start + lo;  // tensor row of this CTA's key 0
  auto issue = [&](int u) {  // producer lane
    const int sl = u % kTdSlots;
    if (u >= kTdSlots) wait(&empty[sl], ((u - kTdSlots) / kTdSlots) & 1);
    unsigned char* dst = ring + (size_t)sl * kTdSlot;
    tcx::mbar_expect_tx(&full[sl], kTdSlot);
    if (u < nq) {
      const int t = u / ns, s = u % ns;
      for (int b = 0; b < 4; ++b)  // box (row half, dim half)
        td_tma2d(dst + b * kTdBox, maps, s * 64 + (b & 1) * 32, y0 + t * kTdKeys + (b >> 1) * 64, &full[sl]);
    } else {
      const int v = u - nq, kb = v / nd, db = v % nd;
      for (int b = 0; b < 4; ++b)  // box = dim quarter
        td_tma2d(dst + b * kTdBox, maps + 128, db * 128 + b * 32, y0 + kb * kTdVKeys, &full[sl]);
    }
  };

  // query planes: tile s (64 dims) = [32 rows][64 B]: row 4h + a = byte a of
  // q_u, row 16 = ones (its products are the key row sums), others zero
  for (int e = tid; e < ns * 32 * 4; e += kTdThreads) {
    const int s = e / 128, rr = (e / 4) % 32, c = e % 4;
    const int h = rr >> 2, limb = rr & 3;
    uint32_t w[4] = {0, 0, 0, 0};
    if (rr < 16 && h < GC) {
      const int4* src = reinterpret_cast<const int4*>(qrow + (size_t)(qh0 + h) * d + s * 64 + c * 16);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int4 v = src[k];
        uint32_t o[4];
        bytes_t4((uint32_t)v.x, (uint32_t)v.y, (uint32_t)v.z, (uint32_t)v.w, o);
        w[k] = o[limb];
      }
    } else if (rr == 16) {
      w[0] = w[1] = w[2] = w[3] = 0x01010101u;
    }
    *reinterpret_cast<uint4*>(qpl + s * 2048 + sw64(rr, c)) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  if (warp < GC) {
    uint64_t t = 0;
    for (int i = lane; i < d; i += 32) t += (uint32_t)qrow[(size_t)(qh0 + warp) * d + i] ^ 0x80000000u;
    t = (uint64_t)td_warp_sum((int64_t)t);
    if (lane == 0) qsum[warp] = t;
  }
  td_fence_async();
  __syncthreads();

  const uint64_t dcorr = (uint64_t)d << 62;
  int32_t bm[GC], bi[GC];
#pragma unroll
  for (int h = 0; h < GC; ++h) { bm[h] = INT32_MIN; bi[h] = INT32_MAX; }

  // epilogue of score tile t (TMEM columns 128 (t & 1) + 32 b + n): epilogue
  // thread of TMEM lane r -> key t*128 + r, every head
  auto score_epilogue = [&](int t) {
    wait(&acc_full[t & 1], (t >> 1) & 1);
    tcx::fence_after();
    const int r = 32 * (warp & 3) + lane;
    const uint32_t taddr = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)(128 * (t & 1));
    uint64_t acc[GC];
#pragma unroll
    for (int h = 0; h < GC; ++h) acc[h] = 0;
    uint64_t ksum = 0;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      uint32_t v[16], one;
      tmem_ld16(taddr + 32 * b, v);
      tmem_ld1(taddr + 32 * b + 16, one);
      tcx::tmem_wait_ld();
      ksum += (uint64_t)one << (8 * b);
#pragma unroll
      for (int h = 0; h < GC; ++h)
#pragma unroll
        for (int l = 0; l < 4; ++l) acc[h] += (uint64_t)v[4 * h + l] << (8 * (b + l));
    }
    const int j = t * kTdKeys + r;  // key index within this CTA
#pragma unroll
    for (int h = 0; h < GC; ++h) {
      if (j < rows) {
        const uint64_t x = acc[h] - (qsum[h] << 31) - (ksum << 31) + dcorr;
        const int32_t s = requantize((int64_t)x);
        sc[h * rmax + j] = s;
        if (s > bm[h] || bi[h] == INT32_MAX) { bm[h] = s; bi[h] = lo + j; }
      }
    }
    tcx::fence_before();
  };

  // ---- scores: the four roles run their own loops, coupled by mbarriers
  if (tid < kTdConv) {
    for (int u = 0; u < nq; ++u) {
      const int pb = u & 1;
      wait(&full[u % kTdSlots], (u / kTdSlots) & 1);
      // key crow's dims 32*half .. +32: box (crow / 64, half), row crow % 64,
      // into registers; the slot goes back to the producer at once
      uint4 w[8];
      {
        const unsigned char* raw = ring + (size_t)(u % kTdSlots) * kTdSlot + ((crow >> 6) * 2 + half) * kTdBox;
        const int br = crow & 63;
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = *reinterpret_cast<const uint4*>(raw + sw128(br, i));
      }
      tcx::mbar_arrive(&empty[u % kTdSlots]);
      if (u >= 2) wait(&mma_done[pb], ((u - 2) >> 1) & 1);
      unsigned char* pl = planes + pb * kTdPlanes;
#pragma unroll
      for (int c = 0; c < 2; ++c) {  // 16-byte output chunk 2*half + c: dims 32*half + 16c ..
        uint32_t o[4][4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          uint32_t q[4];
          bytes_t4(w[4 * c + k].x, w[4 * c + k].y, w[4 * c + k].z, w[4 * c + k].w, q);
#pragma unroll
          for (int b = 0; b < 4; ++b) o[b][k] = q[b];
        }
#pragma unroll
        for (int b = 0; b < 4; ++b)
          *reinterpret_cast<uint4*>(pl + b * kTdPlane + sw64(crow, 2 * half + c)) =
              make_uint4(o[b][0], o[b][1], o[b][2], o[b][3]);
      }
      td_fence_async();
      tcx::mbar_arrive(&planes_full[pb]);
    }
  } else if (warp == kTdProdWarp) {
    if (lane == 0) {
      // the maps were written through the generic proxy (a host copy, possibly
      // into memory that held other maps before): acquire them for the TMA unit
      asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(maps) : "memory");
      asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(maps + 128) : "memory");
      // the score tiles and the first value tiles (these load during the
      // softmax; every slot they reuse held a score tile)
      for (int u = 0; u < total && u < nq + kTdSlots; ++u) issue(u);
    }
  } else if (warp == kTdMmaWarp) {
    if (lane == 0)
      for (int u = 0; u < nq; ++u) {
        const int t = u / ns, s = u % ns, pb = u & 1;
        if (s == 0 && t >= 2) wait(&acc_empty[t & 1], ((t - 2) >> 1) & 1);  // tile t - 2 drained
        wait(&planes_full[pb], (u >> 1) & 1);
        tcx::fence_after();
        const uint32_t pbase = td_su32(planes + pb * kTdPlanes), qbase = td_su32(qpl + s * 2048);
        const uint32_t dcol = tmem + (uint32_t)(128 * (t & 1));
#pragma unroll
        for (int k = 0; k < 2; ++k)
#pragma unroll
          for (int b = 0; b < 4; ++b)
            tcx::mma_i8(dcol + 32 * b, tcx::smem_desc_sw64(pbase + b * kTdPlane + 32 * k),
                        tcx::smem_desc_sw64(qbase + 32 * k), kTdId32, (s > 0 || k > 0) ? 1u : 0u);
        tcx::mma_commit(&mma_done[pb]);
        if (s == ns - 1) tcx::mma_commit(&acc_full[t & 1]);
      }
  } else {
    for (int t = 0; t < ntile; ++t) {
      score_epilogue(t);
      tcx::mbar_arrive(&acc_empty[t & 1]);
    }
  }
  __syncthreads();

  // ---- first max: per head over this CTA, then over the cluster
#pragma unroll
  for (int h = 0; h < GC; ++h) {
    int32_t m = bm[h], mi = bi[h];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const int32_t om = __shfl_xor_sync(0xffffffffu, m, o), oi = __shfl_xor_sync(0xffffffffu, mi, o);
      td_first_max_merge(m, mi, om, oi);
    }
    if (lane == 0) { wm[warp][h] = m; wi[warp][h] = mi; }
  }
  __syncthreads();
  if (tid < GC) {
    int32_t m = INT32_MIN, mi = INT32_MAX;
    for (int w = 0; w < kTdWarps; ++w) td_first_max_merge(m, mi, wm[w][tid], wi[w][tid]);
    s_max[tid] = m;
    s_idx[tid] = mi;
  }
  cl.sync();
  if (warp < GC) {
    int32_t m = INT32_MIN, mi = INT32_MAX;
    if (lane < CL) {
      m = *cl.map_shared_rank(&s_max[warp], lane);
      mi = *cl.map_shared_rank(&s_idx[warp], lane);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const int32_t om = __shfl_xor_sync(0xffffffffu, m, o), oi = __shfl_xor_sync(0xffffffffu, mi, o);
      td_first_max_merge(m, mi, om, oi);
    }
    if (lane == 0) { g_max[warp] = m; g_idx[warp] = mi; }
  }
  __syncthreads();
  // the residual row v[first max] for this CTA's output dims, fetched early
  const int d0 = (int)((int64_t)d * rank / CL), d1 = (int)((int64_t)d * (rank + 1) / CL);
  const int per = d1 - d0;
  for (int e = tid; e < GC * per; e += kTdThreads) {
    const int h = e / per, dim = d0 + e % per;
    td_cp4(&vmx[h][e % per], vc + ((size_t)kvh * capr + start + g_idx[h]) * d + dim);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  // ---- exp terms and local sums (the plane buffers hold the exp terms
  // until the value tiles)
  {
    int64_t sum[GC];
#pragma unroll
    for (int h = 0; h < GC; ++h) sum[h] = 0;
    for (int e = tid; e < GC * rows; e += kTdThreads) {
      const int h = e / rows, j = e - h * rows;
      const int64_t x = exp_term(sc[h * rmax + j], g_max[h]);
      ex[h * rmax + j] = x;
#pragma unroll
      for (int g = 0; g < GC; ++g) sum[g] += g == h ? x : 0;
    }
#pragma unroll
    for (int h = 0; h < GC; ++h) {
      const int64_t t = td_warp_sum(sum[h]);
      if (lane == 0) ws[warp][h] = t;
    }
  }
  __syncthreads();
  if (tid < GC) {
    int64_t t = 0;
    for (int w = 0; w < kTdWarps; ++w) t += ws[w][tid];
    s_sum[tid] = t;
  }
  cl.sync();
  if (warp < GC) {
    const int64_t v = lane < CL ? *cl.map_shared_rank(&s_sum[warp], lane) : 0;
    const int64_t t = td_warp_sum(v);
    if (lane == 0) g_sum[warp] = t;
  }
  __syncthreads();
  // ---- weights and local weight sums
  {
    int64_t wsum[GC];
#pragma unroll
    for (int h = 0; h < GC; ++h) wsum[h] = 0;
    for (int e = tid; e < GC * rows; e += kTdThreads) {
      const int h = e / rows, j = e - h * rows;
      const int32_t w = softmax_weight(ex[h * rmax + j], g_sum[h]);
      sc[h * rmax + j] = w;
#pragma unroll
      for (int g = 0; g < GC; ++g) wsum[g] += g == h ? w : 0;
    }
#pragma unroll
    for (int h = 0; h < GC; ++h) {
      const int64_t t = td_warp_sum(wsum[h]);
      if (lane == 0) ws[warp][h] = t;
    }
  }
  __syncthreads();
  if (tid < GC) {
    int64_t t = 0;
    for (int w = 0; w < kTdWarps; ++w) t += ws[w][tid];
    s_wsum[tid] = t;
  }
  // weight planes: key block kb = [16 rows][64 B], row 4h + a = byte a of w
  // (zero past the CTA's keys, for a = 3 and for h >= GC)
  for (int e = tid; e < nkb * 16 * 4; e += kTdThreads) {
    const int kb = e / 64, rr = (e / 4) % 16, c = e % 4;
    const int h = rr >> 2, limb = rr & 3;
    uint32_t w4[4] = {0, 0, 0, 0};
    if (h < GC && limb < 3) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint32_t bytes = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int j = kb * 64 + c * 16 + 4 * k + i;
          const uint32_t w = j < rows ? (uint32_t)sc[h * rmax + j] : 0u;
          bytes |= ((w >> (8 * limb)) & 0xffu) << (8 * i);
        }
        w4[k] = bytes;
      }
    }
    *reinterpret_cast<uint4*>(wpl + kb * 1024 + sw64(rr, c)) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
  }
  td_fence_async();
  __syncthreads();

  // ---- weighted values: stage v = key block v / nd, dims 128 (v % nd)
  if (tid < kTdConv) {
    for (int u = nq; u < total; ++u) {
      const int pb = u & 1;
      wait(&full[u % kTdSlots], (u / kTdSlots) & 1);
      // dim crow of key rows 32*half .. +32 (box crow / 32, 16-byte chunk
      // (crow % 32) / 4, word crow % 4) into registers; the slot goes back to
      // the producer at once
      uint32_t x[32];
      {
        const unsigned char* raw =
            ring + (size_t)(u % kTdSlots) * kTdSlot + (crow >> 5) * kTdBox + (crow & 3) * 4;
        const int ch = (crow & 31) >> 2;
#pragma unroll
        for (int j = 0; j < 32; ++j) x[j] = *reinterpret_cast<const uint32_t*>(raw + sw128(32 * half + j, ch));
      }
      tcx::mbar_arrive(&empty[u % kTdSlots]);
      if (u >= 2) wait(&mma_done[pb], ((u - 2) >> 1) & 1);
      unsigned char* pl = planes + pb * kTdPlanes;
#pragma unroll
      for (int c = 0; c < 2; ++c) {  // chunk 2*half + c: keys 32*half + 16c ..
        uint32_t o[4][4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int j = 16 * c + 4 * k;
          uint32_t q[4];
          bytes_t4(x[j], x[j + 1], x[j + 2], x[j + 3], q);
#pragma unroll
          for (int b = 0; b < 4; ++b) o[b][k] = q[b];
        }
#pragma unroll
        for (int b = 0; b < 4; ++b)
          *reinterpret_cast<uint4*>(pl + b * kTdPlane + sw64(crow, 2 * half + c)) =
              make_uint4(o[b][0], o[b][1], o[b][2], o[b][3]);
      }
      td_fence_async();
      tcx::mbar_arrive(&planes_full[pb]);
    }
  } else if (warp == kTdProdWarp) {
    if (lane == 0)
      for (int u = nq + kTdSlots; u < total; ++u) issue(u);
  } else if (warp == kTdMmaWarp) {
    if (lane == 0)
      for (int u = nq; u < total; ++u) {
        const int v = u - nq, kb = v / nd, db = v % nd, pb = u & 1;
        wait(&planes_full[pb], (u >> 1) & 1);
        tcx::fence_after();
        const uint32_t pbase = td_su32(planes + pb * kTdPlanes), wbase = td_su32(wpl + kb * 1024);
        const uint32_t dcol = tmem + 256 + (uint32_t)(64 * db);
#pragma unroll
        for (int k = 0; k < 2; ++k)
#pragma unroll
          for (int b = 0; b < 4; ++b)
            tcx::mma_i8(dcol + 16 * b, tcx::smem_desc_sw64(pbase + b * kTdPlane + 32 * k),
                        tcx::smem_desc_sw64(wbase + 32 * k), kTdId16, (kb > 0 || k > 0) ? 1u : 0u);
        tcx::mma_commit(&mma_done[pb]);
        if (u == total - 1) tcx::mma_commit(&pv_full);
      }
  }
  // ---- partial weighted sums of this CTA: lane (dim within a 128-dim block)
  // (pacc overlays the ring: every stage was consumed, the residual row copied)
  // (after the last value MMA every converter read and TMA copy is done, so
  // pacc may overlay the ring)
  if (total > nq && warp >= kTdEpiWarp) {
    wait(&pv_full, 0);
    tcx::fence_after();
    const int r = 32 * (warp & 3) + lane;
    for (int db = 0; db < nd; ++db) {
      const uint32_t taddr = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + 256 + (uint32_t)(64 * db);
      uint64_t acc[GC];
#pragma unroll
      for (int h = 0; h < GC; ++h) acc[h] = 0;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        uint32_t v[16];
        tmem_ld16(taddr + 16 * b, v);
        tcx::tmem_wait_ld();
#pragma unroll
        for (int h = 0; h < GC; ++h)
#pragma unroll
          for (int l = 0; l < 3; ++l) acc[h] += (uint64_t)v[4 * h + l] << (8 * (b + l));
      }
#pragma unroll
      for (int h = 0; h < GC; ++h) pacc[h * d + 128 * db + r] = (int64_t)(acc[h] - ((uint64_t)s_wsum[h] << 31));
    }
  } else if (total == nq) {
    for (int e = tid; e < GC * d; e += kTdThreads) pacc[e] = 0;
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  tcx::fence_before();
  cl.sync();
  // ---- combine: this CTA finalizes output dims [d0, d1)
  if (warp < GC) {
    const int64_t v = lane < CL ? *cl.map_shared_rank(&s_wsum[warp], lane) : 0;
    const int64_t t = td_warp_sum(v);
    if (lane == 0) g_res[warp] = sub_sat(kOneAct, t > INT32_MAX ? INT32_MAX : (int32_t)t);
  }
  __syncthreads();
  const int nel = GC * per, epw = kTdThreads / CL;
  for (int base = 0; base < nel; base += epw) {
    const int e = base + tid / CL, r = tid % CL;
    int64_t v = 0;
    int h = 0, dim = 0;
    if (e < nel) {
      h = e / per;
      dim = d0 + e % per;
      v = *cl.map_shared_rank(&pacc[h * d + dim], r);
    }
    for (int o = CL >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (r == 0 && e < nel) {
      v += (int64_t)vmx[h][dim - d0] * g_res[h];
      orow[(size_t)(qh0 + h) * d + dim] = requantize(v);
    }
  }
  if (s_fail && warp == kTdMmaWarp && lane == 0) {
    atomicExch(&g_tad_err, 1);
    // before the accumulator columns are released: one more bounded wait
    // for this thread's last MMAs
    if (total > nq) tcx::mbar_wait(&pv_full, 0);
    else if (ntile > 0) tcx::mbar_wait(&acc_full[(ntile - 1) & 1], ((ntile - 1) >> 1) & 1);
  }
  tcx::fence_after();
  __syncthreads();
  if (warp == 0) tcx::tmem_dealloc512(tmem);
  cl.sync();  // keep this CTA's shared memory alive until every rank has read it
}

constexpr size_t kTdMaxSmem = 219 * 1024;

template <int GC>
void td_prepare() {
  cudaFuncSetAttribute(attn_dec_tc_kernel<GC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTdMaxSmem);
  cudaFuncSetAttribute(attn_dec_tc_kernel<GC>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
}

template <int GC>
cudaError_t td_launch(const AttnDecodeArgs& a, int CL, int rmax, cudaStream_t s) {
  TdArgs ta;
  ta.a = a;
  ta.rmax = rmax;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(CL, a.Hq / GC, a.batch);
  cfg.blockDim = dim3(kTdThreads, 1, 1);
  cfg.dynamicSmemBytes = td_layout(a.d, rmax, GC).total;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, attn_dec_tc_kernel<GC>, ta);
}

// RDET_TC_DECODE_ATTN=0 selects the CUDA-core kernel (read once per process)
bool td_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("RDET_TC_DECODE_ATTN");
    return !(e && e[0] == '0');
  }();
  return on;
}

}  // namespace

void tc_attn_dec_init() {
  static std::mutex mu;
  static std::vector<char> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  if ((size_t)dev < done.size() && done[dev]) return;
  td_prepare<1>();
  td_prepare<2>();
  td_prepare<4>();
  if ((size_t)dev >= done.size()) done.resize(dev + 1, 0);
  done[dev] = 1;
}

int tc_attn_dec_error_flag(bool reset) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_tad_err, sizeof(int));
  if (reset && v) {
    int z = 0;
    cudaMemcpyToSymbol(g_tad_err, &z, sizeof(int));
  }
  return v;
}

bool td_encode_cache_map(void* out, const int32_t* base, int rows, int d) {
  if (d % 128 != 0 || rows <= 0 || (reinterpret_cast<uintptr_t>(base) & 15) != 0) return false;
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)d, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)d * 4};
  const cuuint32_t box[2] = {32, 64};
  const cuuint32_t estr[2] = {1, 1};
  return fn(reinterpret_cast<CUtensorMap*>(out), CU_TENSOR_MAP_DATA_TYPE_INT32, 2, const_cast<int32_t*>(base), dims,
            strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool launch_attn_decode_tc(const AttnDecodeArgs& a, int sms, cudaStream_t s) {
  if (!td_enabled() || a.batch < 2 || a.fuse.q_in != nullptr || !a.pos_rows || !a.kc_rows || !a.vc_rows ||
      !a.cap_rows || !a.map_rows)
    return false;
  if (a.d % 128 != 0 || a.d > 512) return false;
  const int G = a.group ? a.group : (a.Hkv > 0 ? a.Hq / a.Hkv : 0);
  if (G <= 0) return false;
  const int GC = std::min(G, a.Hq);
  if (!(GC == 1 || GC == 2 || GC == 4) || a.Hq % GC != 0 || G % GC != 0) return false;
  int dev = 0, major = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (major != 10) return false;
  tc_attn_dec_init();
  const int span = a.window > 0 && a.window < a.cap ? a.window : a.cap;
  // at most kTdMaxRows keys and 256 finalized output dims per CTA; among
  // those, clusters that still fill at most one wave
  int CL = 1;
  while (CL < 8 && ((span + CL - 1) / CL > kTdMaxRows || a.d > 256 * CL ||
                    (size_t)td_layout(a.d, (span + CL - 1) / CL + 1, GC).total > kTdMaxSmem))
    CL *= 2;
  const long ctas = (long)a.batch * (a.Hq / GC);
  while (CL < 8 && ctas * CL * 2 <= sms) CL *= 2;
  const int rmax = (span + CL - 1) / CL + 1;
  if (rmax > kTdMaxRows + 1 || a.d > 256 * CL) return false;
  if ((size_t)td_layout(a.d, rmax, GC).total > kTdMaxSmem) return false;
  // launch errors surface through cudaGetLastError in the caller
  if (GC == 1) td_launch<1>(a, CL, rmax, s);
  else if (GC == 2) td_launch<2>(a, CL, rmax, s);
  else td_launch<4>(a, CL, rmax, s);
  return true;
}

}  // namespace rdet
