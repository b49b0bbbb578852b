// det kernels for B200 (sm_100a): GEMV, CUDA-core linear, norms, RoPE,
// attention, embedding, PLE, argmax.  Every kernel computes the reference
// det_num v1 arithmetic exactly (see det_dev.cuh); integer MAC reductions are
// split across lanes/warps/CTAs freely because wrapping i64 addition is
// associative (reference docs/plans/DET_NUM_SPEC.md, "Parallelism legality").
#include <algorithm>
#include <cstdio>
#include <mutex>
#include <vector>

#include <cooperative_groups.h>

#include "det_dev.cuh"
#include "kernels.h"

namespace rdet {

static int g_sms = 0;
int sm_count() {
  if (g_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_sms <= 0) g_sms = 148;
  }
  return g_sms;
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch: every kernel is launched with programmatic
// stream serialization, waits for the grids it depends on to complete (and
// their writes to be visible) before touching their outputs, and lets its own
// dependents start launching right away, so launch latency overlaps the tail
// of the previous kernel.  Launched without the attribute, both are no-ops.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_entry() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
static inline void launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                            Args... args) {
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

// ---------------------------------------------------------------------------
// block reductions
// ---------------------------------------------------------------------------
__device__ __forceinline__ int64_t warp_sum64(int64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
// saturating sum of non-negative i64 terms (order-free: min(true sum, MAX))
__device__ __forceinline__ uint64_t sat_add_u(uint64_t a, uint64_t b) {
  uint64_t s = a + b;
  return (s < a || s > (uint64_t)INT64_MAX) ? (uint64_t)INT64_MAX : s;
}
__device__ __forceinline__ uint64_t warp_satsum(uint64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = sat_add_u(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// rms_norm_scale (ops.rs:406) from each thread's saturating partial sum of
// squares, computed by the whole block; every thread gets the scale.  Warp 0
// combines the per-warp sums (saturating sums are order-free).  `red` is
// >= 33 u64 of smem.
__device__ int32_t block_norm_scale_partial(uint64_t s, int n, int64_t eps, uint64_t* red) {
  s = warp_satsum(s);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = (blockDim.x + 31) >> 5;
  __syncthreads();
  if (l == 0) red[w] = s;
  __syncthreads();
  if (w == 0) {
    const uint64_t t = warp_satsum(l < nw ? red[l] : 0);
    if (l == 0) {
      const int64_t mean = div_acc_by_u32((int64_t)t, (uint32_t)n);
      red[32] = (uint64_t)(uint32_t)inv_sqrt_acc(acc_add_sat(mean, eps));
    }
  }
  __syncthreads();
  return (int32_t)(uint32_t)red[32];
}
// the same over n values in shared memory
__device__ int32_t block_norm_scale(const int32_t* xs, int n, int64_t eps, uint64_t* red) {
  uint64_t s = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s = sat_add_u(s, (uint64_t)mul_wide(xs[i], xs[i]));
  return block_norm_scale_partial(s, n, eps, red);
}
// same for one warp over n values (lane-strided); returns scale to all lanes
__device__ int32_t warp_norm_scale(const int32_t* xs, int n, int64_t eps) {
  uint64_t s = 0;
  for (int i = threadIdx.x & 31; i < n; i += 32) s = sat_add_u(s, (uint64_t)mul_wide(xs[i], xs[i]));
  s = warp_satsum(s);
  int32_t sc = 0;
  if ((threadIdx.x & 31) == 0) sc = inv_sqrt_acc(acc_add_sat(div_acc_by_u32((int64_t)s, (uint32_t)n), eps));
  return __shfl_sync(0xffffffffu, sc, 0);
}

// ---------------------------------------------------------------------------
// decode GEMV
// ---------------------------------------------------------------------------
__device__ __forceinline__ int32_t lo16(uint32_t w) { return (int32_t)(int16_t)(w & 0xffffu); }
__device__ __forceinline__ int32_t hi16(uint32_t w) { return ((int32_t)w) >> 16; }

// Weight streams are read once per token: with an L2 evict-first policy they
// do not push out what is reused within the step (activations, KV rows,
// norm gains, kernel code).
#ifndef RDET_WEIGHTS_EVICT_FIRST
#define RDET_WEIGHTS_EVICT_FIRST 0
#endif
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint4 ldg_stream_pol(const uint4* p, uint64_t pol) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p), "l"(pol));
  return r;
}
__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// dot of one weight row with xs (smem), warp-cooperative, returns the full
// wrapping i64 sum on every lane.
template <int UNR>
__device__ __forceinline__ int64_t row_dot16(const int16_t* row, const int32_t* xs, int K, int lane) {
  int64_t acc = 0;
  if ((K & 7) == 0) {
    const uint4* wr = reinterpret_cast<const uint4*>(row);
    int nc = K >> 3;
    for (int c0 = lane; c0 < nc; c0 += 32 * UNR) {
      uint4 w[UNR];
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        int c = c0 + 32 * u;
        w[u] = c < nc ? ldg_stream(wr + c) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        int c = c0 + 32 * u;
        if (c < nc) {
          const int4* xp = reinterpret_cast<const int4*>(xs + 8 * c);
          int4 a = xp[0], b = xp[1];
          acc = mac_wide(mac_wide(acc, a.x, lo16(w[u].x)), a.y, hi16(w[u].x));
          acc = mac_wide(mac_wide(acc, a.z, lo16(w[u].y)), a.w, hi16(w[u].y));
          acc = mac_wide(mac_wide(acc, b.x, lo16(w[u].z)), b.y, hi16(w[u].z));
          acc = mac_wide(mac_wide(acc, b.z, lo16(w[u].w)), b.w, hi16(w[u].w));
        }
      }
    }
  } else {
    for (int k = lane; k < K; k += 32) acc = mac_wide(acc, xs[k], (int32_t)row[k]);
  }
  return warp_sum64(acc);
}
template <int UNR>
__device__ __forceinline__ int64_t row_dot32(const int32_t* row, const int32_t* xs, int K, int lane) {
  int64_t acc = 0;
  if ((K & 3) == 0) {
    const uint4* wr = reinterpret_cast<const uint4*>(row);
    int nc = K >> 2;
    for (int c0 = lane; c0 < nc; c0 += 32 * UNR) {
      uint4 w[UNR];
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        int c = c0 + 32 * u;
        w[u] = c < nc ? ldg_stream(wr + c) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        int c = c0 + 32 * u;
        if (c < nc) {
          int4 a = reinterpret_cast<const int4*>(xs)[c];
          acc = mac_wide(mac_wide(acc, a.x, (int32_t)w[u].x), a.y, (int32_t)w[u].y);
          acc = mac_wide(mac_wide(acc, a.z, (int32_t)w[u].z), a.w, (int32_t)w[u].w);
        }
      }
    }
  } else {
    for (int k = lane; k < K; k += 32) acc = mac_wide(acc, xs[k], (int32_t)row[k]);
  }
  return warp_sum64(acc);
}
__device__ __forceinline__ int64_t mat_row_dot(const DevMat& m, int r, const int32_t* xs, int K, int lane) {
  if (m.width == 16) return row_dot16<8>(static_cast<const int16_t*>(m.p) + (size_t)r * K, xs, K, lane);
  return row_dot32<8>(static_cast<const int32_t*>(m.p) + (size_t)r * K, xs, K, lane);
}

constexpr int kGemvThreads = 256;

__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const GemvArgs a) {
  pdl_entry();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int32_t* xs = reinterpret_cast<int32_t*>(smem_raw);
  __shared__ uint64_t red[33];
  const int K = a.K;
  // ---- prologue: build x in shared memory
  for (int i = threadIdx.x; i < K; i += blockDim.x) xs[i] = a.a[i];
  __syncthreads();
  if (a.pro != kProNone) {
    int32_t sc = block_norm_scale(xs, K, a.eps, red);
    if (a.pro == kProNorm) {
      for (int i = threadIdx.x; i < K; i += blockDim.x) xs[i] = mul_sat(mul_sat(xs[i], sc), a.g1[i]);
    } else {
      for (int i = threadIdx.x; i < K; i += blockDim.x) {
        int32_t t = add_sat(a.res[i], mul_sat(mul_sat(xs[i], sc), a.g1[i]));
        if (a.has_scalar) t = mul_sat(t, a.scalar);
        xs[i] = t;
        if (blockIdx.x == 0 && a.t_out) a.t_out[i] = t;
      }
      __syncthreads();
      if (a.pro == kProResNorm || a.pro == kProResScaleNorm) {
        int32_t sc2 = block_norm_scale(xs, K, a.eps, red);
        for (int i = threadIdx.x; i < K; i += blockDim.x) xs[i] = mul_sat(mul_sat(xs[i], sc2), a.g2[i]);
      }
    }
  }
  __syncthreads();
  // ---- rows
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const int gw = blockIdx.x * warps + (threadIdx.x >> 5);
  const int nw = gridDim.x * warps;
  if (a.pair_geglu) {
    const int R = a.seg[0].w.rows;
    for (int r = gw; r < R; r += nw) {
      int64_t g = mat_row_dot(a.seg[0].w, r, xs, K, lane);
      int64_t u = mat_row_dot(a.seg[1].w, r, xs, K, lane);
      if (lane == 0) a.seg[0].y[r] = mul_sat(gelu_act(requantize(g)), requantize(u));
    }
    return;
  }
  int total = 0;
  for (int s = 0; s < a.nseg; ++s) total += a.seg[s].w.rows;
  for (int gr = gw; gr < total; gr += nw) {
    int s = 0, r = gr;
    while (r >= a.seg[s].w.rows) { r -= a.seg[s].w.rows; ++s; }
    const GemvSeg& sg = a.seg[s];
    int64_t acc = mat_row_dot(sg.w, r, xs, K, lane);
    if (lane == 0) {
      int32_t v = requantize(acc);
      if (sg.epi == kEpiSoftcap) v = softcap_act(v, a.softcap);
      else if (sg.epi == kEpiGeluMul) v = mul_sat(gelu_act(v), sg.vec[r]);
      sg.y[r] = v;
    }
  }
}

// ---------------------------------------------------------------------------
// decode GEMV v2: weights streamed with bulk async copies (cp.async.bulk) into
// an mbarrier-pipelined ring of shared-memory stages.  One persistent CTA per
// SM owns a balanced slice of rows of every matrix in the launch; a producer
// warp streams whole rows (contiguous in HBM) while 8 consumer warps do the
// exact i64 MACs from shared memory.  Per-row partial sums are combined in
// shared memory with wrapping 64-bit adds (order-free), then requantized once.
// Every pipeline wait is bounded: on timeout the kernel records the failure
// in g_stream_err and returns instead of hanging.
// ---------------------------------------------------------------------------
__device__ int g_stream_err = 0;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// bounded wait on an mbarrier phase (each try_wait may suspend the thread
// for a hardware-defined interval, so the bound is a few seconds at most)
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity) {
  for (uint32_t i = 0; i < (1u << 22); ++i)
    if (mbar_test(b, parity)) return true;
  return false;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}


// Shape of the streamed GEMV (compile-time tunables).
#ifndef RDET_STREAM_CONSUMER_WARPS
#define RDET_STREAM_CONSUMER_WARPS 8
#endif
#ifndef RDET_STREAM_STAGE_BYTES
#define RDET_STREAM_STAGE_BYTES (24 * 1024)
#endif
#ifndef RDET_STREAM_CTAS_PER_SM
#define RDET_STREAM_CTAS_PER_SM 1
#endif
#ifndef RDET_STREAM_MAX_STAGES
#define RDET_STREAM_MAX_STAGES 8
#endif
constexpr int kStreamConsumerWarps = RDET_STREAM_CONSUMER_WARPS;
constexpr int kStreamConsumerThreads = 32 * kStreamConsumerWarps;
constexpr int kStreamThreads = 32 * (kStreamConsumerWarps + 1);
constexpr int kStreamMaxStages = RDET_STREAM_MAX_STAGES;
constexpr int kStreamCtasPerSm = RDET_STREAM_CTAS_PER_SM;

struct StreamCfg {
  int ns;              // pipeline stages
  int stage_bytes;     // bytes per stage buffer
  int rs[3];           // rows per stage, per job
  int acc_off[3];      // accumulator offset (rows) per job
  int rpc[3];          // max rows per CTA per job
  int njobs;
  int x_bytes;         // bytes of the x buffer (K*4, rounded up to 128)
};

__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync 1, %0;" ::"r"(kStreamConsumerThreads) : "memory");
}

// rms scale over the consumer threads (x in permuted layout; the sum is order-free)
__device__ int32_t consumer_norm_scale(const int32_t* xs, int n, int64_t eps, uint64_t* red) {
  uint64_t s = 0;
  for (int i = threadIdx.x; i < n; i += kStreamConsumerThreads) {
    int64_t v = xs[i];
    s = sat_add_u(s, (uint64_t)(v * v));
  }
  s = warp_satsum(s);
  consumers_sync();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  consumers_sync();
  if (threadIdx.x == 0) {
    uint64_t t = 0;
    for (int i = 0; i < kStreamConsumerWarps; ++i) t = sat_add_u(t, red[i]);
    red[32] = (uint64_t)(uint32_t)inv_sqrt_acc(acc_add_sat(div_acc_by_u32((int64_t)t, (uint32_t)n), eps));
  }
  consumers_sync();
  return (int32_t)(uint32_t)red[32];
}

template <int WB>  // weight bytes: 2 (i16) or 4 (i32)
__global__ void __launch_bounds__(kStreamThreads, kStreamCtasPerSm) gemv_stream_kernel(const GemvArgs a,
                                                                                       const StreamCfg cfg) {
  pdl_entry();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t full[kStreamMaxStages], empty[kStreamMaxStages];
  __shared__ uint64_t red[33];
  const int K = a.K;
  int32_t* xs = reinterpret_cast<int32_t*>(smem_raw);                      // x in chunk-plane layout
  unsigned char* stages = smem_raw + cfg.x_bytes;
  int64_t* acc = reinterpret_cast<int64_t*>(stages + (size_t)cfg.ns * cfg.stage_bytes);
  const int G = gridDim.x, cta = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rowbytes = K * WB;
  const int KC = rowbytes / 16;  // 16-byte chunks per row
  if (threadIdx.x == 0) {
    for (int i = 0; i < cfg.ns; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kStreamConsumerWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == kStreamConsumerWarps) {
    // ---------------- producer: stream this CTA's rows of every job
    if (lane == 0) {
      int t = 0;
      bool ok = true;
      for (int j = 0; j < cfg.njobs && ok; ++j) {
        const int N = a.seg[j].w.rows;
        const int lo = (int)((int64_t)N * cta / G), hi = (int)((int64_t)N * (cta + 1) / G);
        const unsigned char* W = static_cast<const unsigned char*>(a.seg[j].w.p);
        for (int r = lo; r < hi; r += cfg.rs[j], ++t) {
          const int s = t % cfg.ns, k = t / cfg.ns;
          if (t >= cfg.ns && !mbar_wait(&empty[s], (k - 1) & 1)) { ok = false; break; }
          const int nr = min(cfg.rs[j], hi - r);
          const uint32_t bytes = (uint32_t)nr * rowbytes;
          mbar_arrive_tx(&full[s], bytes);
          bulk_g2s(stages + (size_t)s * cfg.stage_bytes, W + (size_t)r * rowbytes, bytes, &full[s]);
        }
      }
      if (!ok) {
        atomicExch(&g_stream_err, 1);
        // let the copies already issued land before the CTA's shared memory goes away
        for (int i = 0; i < cfg.ns; ++i) {
          int tt = t - 1 - i;
          if (tt < 0) break;
          mbar_wait(&full[tt % cfg.ns], (tt / cfg.ns) & 1);
        }
      }
    }
    return;
  }

  // ---------------- consumers: prologue builds x (permuted chunk layout for i16)
  // storage index p <-> element e: for i16, chunk c = e/8 has its low half at
  // plane 0 [c*4 ..] and high half at plane 1 [K/2 + c*4 ..] (conflict-free LDS.128)
  auto elem = [&](int p) -> int {
    if (WB == 4) return p;
    int h = p >= (K >> 1);
    int q = p - h * (K >> 1);
    return (q >> 2) * 8 + h * 4 + (q & 3);
  };
  for (int p = threadIdx.x; p < K; p += kStreamConsumerThreads) xs[p] = a.a[elem(p)];
  for (int j = 0; j < cfg.njobs; ++j)
    for (int i = threadIdx.x; i < cfg.rpc[j]; i += kStreamConsumerThreads) acc[cfg.acc_off[j] + i] = 0;
  consumers_sync();
  if (a.pro != kProNone) {
    int32_t sc = consumer_norm_scale(xs, K, a.eps, red);
    if (a.pro == kProNorm) {
      for (int p = threadIdx.x; p < K; p += kStreamConsumerThreads) xs[p] = mul_sat(mul_sat(xs[p], sc), a.g1[elem(p)]);
    } else {
      for (int p = threadIdx.x; p < K; p += kStreamConsumerThreads) {
        int e = elem(p);
        int32_t t = add_sat(a.res[e], mul_sat(mul_sat(xs[p], sc), a.g1[e]));
        if (a.has_scalar) t = mul_sat(t, a.scalar);
        xs[p] = t;
        if (cta == 0 && a.t_out) a.t_out[e] = t;
      }
      consumers_sync();
      if (a.pro == kProResNorm || a.pro == kProResScaleNorm) {
        int32_t sc2 = consumer_norm_scale(xs, K, a.eps, red);
        for (int p = threadIdx.x; p < K; p += kStreamConsumerThreads) xs[p] = mul_sat(mul_sat(xs[p], sc2), a.g2[elem(p)]);
      }
    }
  }
  consumers_sync();

  // ---------------- consumers: stages
  bool ok = true;
  int t = 0;
  for (int j = 0; j < cfg.njobs && ok; ++j) {
    const int N = a.seg[j].w.rows;
    const int lo = (int)((int64_t)N * cta / G), hi = (int)((int64_t)N * (cta + 1) / G);
    int64_t* accj = acc + cfg.acc_off[j];
    for (int r = lo; r < hi; r += cfg.rs[j], ++t) {
      const int s = t % cfg.ns, k = t / cfg.ns;
      if (!mbar_wait(&full[s], k & 1)) { ok = false; break; }
      const int nr = min(cfg.rs[j], hi - r);
      const int C = nr * KC;
      const int c0 = (int)((int64_t)C * warp / kStreamConsumerWarps);
      const int c1 = (int)((int64_t)C * (warp + 1) / kStreamConsumerWarps);
      const uint4* sp = reinterpret_cast<const uint4*>(stages + (size_t)s * cfg.stage_bytes);
      int c = c0 + lane;
      int row = c / KC, col = c - row * KC;
      int cur_row = -1;
      int64_t cur = 0;
      for (; c < c1; c += 32) {
        uint4 w = sp[c];
        int64_t p;
        if (WB == 2) {
          int4 xa = reinterpret_cast<const int4*>(xs)[col];
          int4 xb = reinterpret_cast<const int4*>(xs + (K >> 1))[col];
          p = (int64_t)xa.x * lo16(w.x) + (int64_t)xa.y * hi16(w.x) + (int64_t)xa.z * lo16(w.y) +
              (int64_t)xa.w * hi16(w.y) + (int64_t)xb.x * lo16(w.z) + (int64_t)xb.y * hi16(w.z) +
              (int64_t)xb.z * lo16(w.w) + (int64_t)xb.w * hi16(w.w);
        } else {
          int4 xa = reinterpret_cast<const int4*>(xs)[col];
          p = (int64_t)xa.x * (int32_t)w.x + (int64_t)xa.y * (int32_t)w.y + (int64_t)xa.z * (int32_t)w.z +
              (int64_t)xa.w * (int32_t)w.w;
        }
        if (row != cur_row) {
          if (cur_row >= 0) atomicAdd(reinterpret_cast<unsigned long long*>(&accj[r - lo + cur_row]), (unsigned long long)cur);
          cur_row = row;
          cur = p;
        } else {
          cur += p;
        }
        col += 32;
        while (col >= KC) { col -= KC; ++row; }
      }
      const int r0 = __shfl_sync(0xffffffffu, cur_row, 0);
      if (__all_sync(0xffffffffu, cur_row == r0)) {
        int64_t tot = warp_sum64(cur);
        if (lane == 0 && r0 >= 0) atomicAdd(reinterpret_cast<unsigned long long*>(&accj[r - lo + r0]), (unsigned long long)tot);
      } else if (cur_row >= 0) {
        atomicAdd(reinterpret_cast<unsigned long long*>(&accj[r - lo + cur_row]), (unsigned long long)cur);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
  }
  if (!ok) {
    atomicExch(&g_stream_err, 1);
    return;
  }
  consumers_sync();
  // ---------------- epilogue
  if (a.pair_geglu) {
    const int N = a.seg[0].w.rows;
    const int lo = (int)((int64_t)N * cta / G), hi = (int)((int64_t)N * (cta + 1) / G);
    for (int r = lo + threadIdx.x; r < hi; r += kStreamConsumerThreads)
      a.seg[0].y[r] = mul_sat(gelu_act(requantize(acc[cfg.acc_off[0] + r - lo])), requantize(acc[cfg.acc_off[1] + r - lo]));
    return;
  }
  for (int j = 0; j < cfg.njobs; ++j) {
    const GemvSeg& sg = a.seg[j];
    const int N = sg.w.rows;
    const int lo = (int)((int64_t)N * cta / G), hi = (int)((int64_t)N * (cta + 1) / G);
    for (int r = lo + threadIdx.x; r < hi; r += kStreamConsumerThreads) {
      int32_t v = requantize(acc[cfg.acc_off[j] + r - lo]);
      if (sg.epi == kEpiSoftcap) v = softcap_act(v, a.softcap);
      else if (sg.epi == kEpiGeluMul) v = mul_sat(gelu_act(v), sg.vec[r]);
      sg.y[r] = v;
    }
  }
}

static void stream_set_attrs() {
  cudaFuncSetAttribute(gemv_stream_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
  cudaFuncSetAttribute(gemv_stream_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
}
static void attn_cluster_init();
// Function attributes are per device: set them once for each device.
void kernels_init() {
  static std::mutex mu;
  static std::vector<char> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  if ((size_t)dev < done.size() && done[dev]) return;
  stream_set_attrs();
  attn_cluster_init();
  tc_init();
  tc_attn_init();
  if ((size_t)dev >= done.size()) done.resize(dev + 1, 0);
  done[dev] = 1;
}

int stream_error_flag(bool reset) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_stream_err, sizeof(int));
  if (reset && v) {
    int z = 0;
    cudaMemcpyToSymbol(g_stream_err, &z, sizeof(int));
  }
  return v | tc_error_flag(reset) | tc_attn_error_flag(reset) | tc_attn_dec_error_flag(reset);
}

// Plans and launches the streamed GEMV; returns false when the launch does not
// qualify (mixed widths, unaligned rows, oversize rows), so v1 runs instead.
[[maybe_unused]] static bool launch_gemv_stream(const GemvArgs& a, cudaStream_t s) {
  const int njobs = a.pair_geglu ? 2 : a.nseg;
  const int width = a.seg[0].w.width;
  for (int j = 0; j < njobs; ++j) {
    if (a.seg[j].w.width != width || a.seg[j].w.cols != a.K) return false;
    if ((reinterpret_cast<uintptr_t>(a.seg[j].w.p) & 15) != 0) return false;
  }
  const int WB = width / 8;
  const long rowbytes = (long)a.K * WB;
  if (rowbytes % 16 != 0 || rowbytes > 48 * 1024) return false;
  if (WB == 2 && (a.K % 16) != 0) return false;  // chunk planes need K/2 divisible by 8
  const int G = sm_count() * kStreamCtasPerSm;
  StreamCfg cfg{};
  cfg.njobs = njobs;
  cfg.x_bytes = (int)(((long)a.K * 4 + 127) / 128 * 128);
  int acc_rows = 0;
  for (int j = 0; j < njobs; ++j) {
    const int N = a.seg[j].w.rows;
    cfg.rpc[j] = (N + G - 1) / G + 1;
    cfg.acc_off[j] = acc_rows;
    acc_rows += cfg.rpc[j];
  }
  const long acc_bytes = (long)acc_rows * 8;
  const long budget = 216L * 1024 / kStreamCtasPerSm - cfg.x_bytes - acc_bytes;
  const long target = RDET_STREAM_STAGE_BYTES;
  long stage = rowbytes >= target ? rowbytes : (target / rowbytes) * rowbytes;
  int ns = (int)(budget / stage);
  if (ns > kStreamMaxStages) ns = kStreamMaxStages;
  if (ns < 2) return false;
  cfg.ns = ns;
  cfg.stage_bytes = (int)((stage + 127) / 128 * 128);
  for (int j = 0; j < njobs; ++j) cfg.rs[j] = (int)(stage / rowbytes);
  const size_t smem = (size_t)cfg.x_bytes + (size_t)cfg.ns * cfg.stage_bytes + (size_t)acc_bytes;
  if (smem > 220 * 1024 / kStreamCtasPerSm) return false;
  stream_set_attrs();
  if (WB == 2) launch_k(gemv_stream_kernel<2>, dim3(G), dim3(kStreamThreads), smem, s, a, cfg);
  else launch_k(gemv_stream_kernel<4>, dim3(G), dim3(kStreamThreads), smem, s, a, cfg);
  return true;
}

// ---------------------------------------------------------------------------
// decode GEMV v3: each warp computes two rows at once (for gate/up, the gate
// row and the up row of the same output), all loads of a row piece issued
// before any math, and four independent i64 accumulator chains.
// ---------------------------------------------------------------------------
#ifndef RDET_GEMV3_NCH
#define RDET_GEMV3_NCH 10
#endif
// Two shapes of the same kernel: 256 threads x 2 CTAs per SM, and 512 x 1.
// Every CTA builds the input vector itself; the 512-thread shape halves that
// redundant prologue work per SM and measured fastest over a whole decode
// step, so the launcher uses it throughout.
constexpr int kG3ThreadsPerSm = 512;
#ifndef RDET_GEMV3_NCH_W32
#define RDET_GEMV3_NCH_W32 6
#endif

// (The product form (int64_t)x * w is kept here: the streaming GEMV is
// bound by HBM, and mac_wide chains raised its register use past the
// 512-thread budget.)
template <int WB>
__device__ __forceinline__ void dot_chunk(const uint4& w, const int32_t* xs, int c, int64_t& a0, int64_t& a1) {
  if (WB == 2) {
    const int4* xp = reinterpret_cast<const int4*>(xs + 8 * c);
    int4 x0 = xp[0], x1 = xp[1];
    a0 += (int64_t)x0.x * lo16(w.x);
    a1 += (int64_t)x0.y * hi16(w.x);
    a0 += (int64_t)x0.z * lo16(w.y);
    a1 += (int64_t)x0.w * hi16(w.y);
    a0 += (int64_t)x1.x * lo16(w.z);
    a1 += (int64_t)x1.y * hi16(w.z);
    a0 += (int64_t)x1.z * lo16(w.w);
    a1 += (int64_t)x1.w * hi16(w.w);
  } else {
    int4 x0 = reinterpret_cast<const int4*>(xs)[c];
    a0 += (int64_t)x0.x * (int32_t)w.x;
    a1 += (int64_t)x0.y * (int32_t)w.y;
    a0 += (int64_t)x0.z * (int32_t)w.z;
    a1 += (int64_t)x0.w * (int32_t)w.w;
  }
}

// Row-pair pieces: a piece is the next kG3Nch 16-byte chunks per lane of two
// rows.  Loads of a piece are issued together, then consumed.
template <int WB>
struct G3Piece {
  static constexpr int N = WB == 2 ? RDET_GEMV3_NCH : RDET_GEMV3_NCH_W32;
  uint4 wa[N], wb[N];
};
template <int WB>
__device__ __forceinline__ void g3_load(G3Piece<WB>& p, const uint4* pa, const uint4* pb, bool has_b, int c0, int nc,
                                        uint64_t pol) {
#pragma unroll
  for (int u = 0; u < G3Piece<WB>::N; ++u) {
    int c = c0 + 32 * u;
#if RDET_WEIGHTS_EVICT_FIRST
    p.wa[u] = c < nc ? ldg_stream_pol(pa + c, pol) : make_uint4(0, 0, 0, 0);
    p.wb[u] = (has_b && c < nc) ? ldg_stream_pol(pb + c, pol) : make_uint4(0, 0, 0, 0);
#else
    p.wa[u] = c < nc ? ldg_stream(pa + c) : make_uint4(0, 0, 0, 0);
    p.wb[u] = (has_b && c < nc) ? ldg_stream(pb + c) : make_uint4(0, 0, 0, 0);
#endif
  }
}
template <int WB>
__device__ __forceinline__ void g3_consume(const G3Piece<WB>& p, const int32_t* xs, bool has_b, int c0, int nc,
                                           int64_t& a0, int64_t& a1, int64_t& b0, int64_t& b1) {
#pragma unroll
  for (int u = 0; u < G3Piece<WB>::N; ++u) {
    int c = c0 + 32 * u;
    if (c < nc) {
      dot_chunk<WB>(p.wa[u], xs, c, a0, a1);
      if (has_b) dot_chunk<WB>(p.wb[u], xs, c, b0, b1);
    }
  }
}

// Work item `gp` -> (matrix A row ra, matrix B row rb, has_b, segment)
struct G3Item {
  const unsigned char* A;
  const unsigned char* B;
  int ra, rb, seg;
  bool has_b;
};
__device__ __forceinline__ G3Item g3_item(const GemvArgs& a, int gp, int per_item) {
  G3Item it;
  if (a.pair_geglu) {
    it.A = static_cast<const unsigned char*>(a.seg[0].w.p);
    it.B = static_cast<const unsigned char*>(a.seg[1].w.p);
    it.ra = it.rb = gp;
    it.seg = 0;
    it.has_b = true;
    return it;
  }
  int sgi = 0, p = gp;
  for (;;) {
    int pr = (a.seg[sgi].w.rows + per_item - 1) / per_item;
    if (p < pr) break;
    p -= pr;
    ++sgi;
  }
  it.A = it.B = static_cast<const unsigned char*>(a.seg[sgi].w.p);
  it.ra = per_item * p;
  it.rb = it.ra + 1;
  it.has_b = per_item == 2 && it.rb < a.seg[sgi].w.rows;
  it.seg = sgi;
  return it;
}

__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(sa), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// K ints into shared memory, 4-byte copies through L1 (measured faster here
// than 16-byte L1-bypassing copies for vectors the previous kernel wrote).
__device__ __forceinline__ void g3_vec_load(int32_t* dst, const int32_t* src, int K) {
  for (int i = threadIdx.x; i < K; i += blockDim.x) cp_async4(dst + i, src + i);
}

// Shared-memory vectors of the GEMV prologue, each K ints: x, then (when the
// prologue uses them) res, g1, g2.
__host__ __device__ inline int gemv_pro_vectors(int pro) {
  switch (pro) {
    case kProNorm: return 2;
    case kProResScale: return 3;
    case kProResNorm:
    case kProResScaleNorm: return 4;
    default: return 1;
  }
}

template <int WB>
__device__ __forceinline__ void g3_epilogue(const GemvArgs& a, const G3Item& it, int lane, int64_t da, int64_t db) {
  if (a.pair_geglu) {
    if (lane == 0) a.seg[0].y[it.ra] = mul_sat(gelu_act(requantize(da)), requantize(db));
    return;
  }
  const GemvSeg& sg = a.seg[it.seg];
  if (lane < 2 && (lane == 0 || it.has_b)) {
    const int r = lane == 0 ? it.ra : it.rb;
    int32_t v = requantize(lane == 0 ? da : db);
    if (sg.epi == kEpiSoftcap) v = softcap_act(v, a.softcap);
    else if (sg.epi == kEpiGeluMul) v = mul_sat(gelu_act(v), sg.vec[r]);
    sg.y[r] = v;
  }
}

template <int WB, int THREADS>
__global__ void __launch_bounds__(THREADS, kG3ThreadsPerSm / THREADS) gemv3_kernel(const GemvArgs a, int per_item) {
  // Weights and norm gains never depend on earlier kernels: the first piece
  // of this warp's first item and the gains are requested before waiting on
  // the preceding grid.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const uint64_t pol = l2_evict_first_policy();
  const int K = a.K;
  int32_t* xs = reinterpret_cast<int32_t*>(smem_raw);
  int32_t* rs = xs + K;
  int32_t* g1s = a.pro == kProNorm ? xs + K : rs + K;
  int32_t* g2s = g1s + K;
  __shared__ uint64_t red[33];
  const int nc = K * WB / 16;
  const int lane = threadIdx.x & 31;
  // items go round the CTAs first (item i -> CTA i % grid), so a GEMV with
  // fewer items than warp slots still streams from every SM
  const int gw = (threadIdx.x >> 5) * gridDim.x + blockIdx.x;
  const int nw = gridDim.x * (blockDim.x >> 5);
  const bool has_res = a.pro == kProResNorm || a.pro == kProResScale || a.pro == kProResScaleNorm;
  const bool norm2 = a.pro == kProResNorm || a.pro == kProResScaleNorm;
  int total = 0;
  if (a.pair_geglu) total = a.seg[0].w.rows;
  else for (int j = 0; j < a.nseg; ++j) total += (a.seg[j].w.rows + per_item - 1) / per_item;
  G3Piece<WB> pc;
  G3Item it;
  const uint4 *pa = nullptr, *pb = nullptr;
  if (gw < total) {
    it = g3_item(a, gw, per_item);
    pa = reinterpret_cast<const uint4*>(it.A + (size_t)it.ra * K * WB);
    pb = reinterpret_cast<const uint4*>(it.B + (size_t)(it.has_b ? it.rb : it.ra) * K * WB);
    g3_load<WB>(pc, pa, pb, it.has_b, lane, nc, pol);
  }
  if (a.pro != kProNone) g3_vec_load(g1s, a.g1, K);
  if (norm2) g3_vec_load(g2s, a.g2, K);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  g3_vec_load(xs, a.a, K);
  if (has_res) g3_vec_load(rs, a.res, K);
  cp_async_wait_all();
  __syncthreads();
  if (a.pro != kProNone) {
    int32_t sc = block_norm_scale(xs, K, a.eps, red);
    if (a.pro == kProNorm) {
      for (int i = threadIdx.x; i < K; i += blockDim.x) xs[i] = mul_sat(mul_sat(xs[i], sc), g1s[i]);
    } else {
      // the residual pass also gathers the squares the second norm needs;
      // each thread rescales only the elements it wrote
      uint64_t s2 = 0;
      for (int i = threadIdx.x; i < K; i += blockDim.x) {
        int32_t t = add_sat(rs[i], mul_sat(mul_sat(xs[i], sc), g1s[i]));
        if (a.has_scalar) t = mul_sat(t, a.scalar);
        xs[i] = t;
        s2 = sat_add_u(s2, (uint64_t)mul_wide(t, t));
        if (blockIdx.x == 0 && a.t_out) a.t_out[i] = t;
      }
      if (norm2) {
        const int32_t sc2 = block_norm_scale_partial(s2, K, a.eps, red);
        for (int i = threadIdx.x; i < K; i += blockDim.x) xs[i] = mul_sat(mul_sat(xs[i], sc2), g2s[i]);
      }
    }
  }
  __syncthreads();
  // The first piece of every item is already in flight when the item starts:
  // the next item's is issued before this item's epilogue.
  for (int gp = gw; gp < total;) {
    int64_t a0 = 0, a1 = 0, b0 = 0, b1 = 0;
    for (int c0 = lane; c0 < nc; c0 += 32 * G3Piece<WB>::N) {
      if (c0 != lane) g3_load<WB>(pc, pa, pb, it.has_b, c0, nc, pol);
      g3_consume<WB>(pc, xs, it.has_b, c0, nc, a0, a1, b0, b1);
    }
    const int64_t da = warp_sum64(a0 + a1), db = warp_sum64(b0 + b1);
    const G3Item cur = it;
    const int gn = gp + nw;
    if (gn < total) {
      it = g3_item(a, gn, per_item);
      pa = reinterpret_cast<const uint4*>(it.A + (size_t)it.ra * K * WB);
      pb = reinterpret_cast<const uint4*>(it.B + (size_t)(it.has_b ? it.rb : it.ra) * K * WB);
      g3_load<WB>(pc, pa, pb, it.has_b, lane, nc, pol);
    }
    g3_epilogue<WB>(a, cur, lane, da, db);
    gp = gn;
  }
}

static bool launch_gemv3(const GemvArgs& a, cudaStream_t s) {
  const int njobs = a.pair_geglu ? 2 : a.nseg;
  const int width = a.seg[0].w.width;
  for (int j = 0; j < njobs; ++j) {
    if (a.seg[j].w.width != width || a.seg[j].w.cols != a.K) return false;
    if ((reinterpret_cast<uintptr_t>(a.seg[j].w.p) & 15) != 0) return false;
  }
  const int WB = width / 8;
  if (((long)a.K * WB) % 16 != 0) return false;
  int rows = 0;
  for (int j = 0; j < a.nseg; ++j) rows += a.seg[j].w.rows;
  const int threads = 512;
  // two rows per warp item unless that would leave most warp slots idle
  const int warps = threads / 32;
  const int cap = sm_count() * (kG3ThreadsPerSm / threads);
  const int per_item = (!a.pair_geglu && rows < cap * warps) ? 1 : 2;
  int items = 0;
  if (a.pair_geglu) items = a.seg[0].w.rows;
  else for (int j = 0; j < a.nseg; ++j) items += (a.seg[j].w.rows + per_item - 1) / per_item;
  int blocks = items;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  const size_t smem = (size_t)a.K * 4 * gemv_pro_vectors(a.pro);
  if (smem > 200 * 1024) return false;
  if (smem > 48 * 1024) {
    cudaFuncSetAttribute(gemv3_kernel<2, 256>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaFuncSetAttribute(gemv3_kernel<4, 256>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaFuncSetAttribute(gemv3_kernel<2, 512>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaFuncSetAttribute(gemv3_kernel<4, 512>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  }
  const dim3 grid(blocks), block(threads);
  if (WB == 2) {
    if (threads == 512) launch_k(gemv3_kernel<2, 512>, grid, block, smem, s, a, per_item);
    else launch_k(gemv3_kernel<2, 256>, grid, block, smem, s, a, per_item);
  } else {
    if (threads == 512) launch_k(gemv3_kernel<4, 512>, grid, block, smem, s, a, per_item);
    else launch_k(gemv3_kernel<4, 256>, grid, block, smem, s, a, per_item);
  }
  return true;
}

void launch_gemv(const GemvArgs& a, cudaStream_t s) {
#ifdef RDET_GEMV_STREAMED
  if (launch_gemv_stream(a, s)) return;
#else
  if (launch_gemv3(a, s)) return;
#endif
  int rows = 0;
  if (a.pair_geglu) rows = a.seg[0].w.rows;
  else for (int i = 0; i < a.nseg; ++i) rows += a.seg[i].w.rows;
  int warps = kGemvThreads / 32;
  int blocks = (rows + warps - 1) / warps;
  int cap = sm_count() * 4;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  size_t smem = (size_t)a.K * 4;
  if (smem > 48 * 1024) cudaFuncSetAttribute(gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  launch_k(gemv_kernel, dim3(blocks), dim3(kGemvThreads), smem, s, a);
}

// ---------------------------------------------------------------------------
// prefill linear on CUDA cores: Y[S,N] = requantize(X[S,K] W[N,K]^T)
// 64x64 output tile, 256 threads, 4x4 i64 accumulators per thread.
// ---------------------------------------------------------------------------
constexpr int LT_BM = 64, LT_BN = 64, LT_BK = 32;

template <bool PAIR>
__global__ void __launch_bounds__(256) linear_kernel(const int32_t* __restrict__ X, int S, DevMat w, DevMat wu,
                                                     int32_t* __restrict__ Y, int epi, const int32_t* __restrict__ vec) {
  pdl_entry();
  __shared__ int32_t xs[LT_BK][LT_BM + 1];
  __shared__ int32_t ws[LT_BK][LT_BN + 1];
  __shared__ int32_t us[PAIR ? LT_BK : 1][PAIR ? LT_BN + 1 : 1];
  const int N = w.rows, K = w.cols;
  const int s0 = blockIdx.y * LT_BM, n0 = blockIdx.x * LT_BN;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  int64_t acc[4][4] = {};
  int64_t accu[PAIR ? 4 : 1][PAIR ? 4 : 1] = {};
  for (int k0 = 0; k0 < K; k0 += LT_BK) {
    for (int e = threadIdx.x; e < LT_BM * LT_BK; e += 256) {
      int r = e / LT_BK, c = e % LT_BK;
      int gs = s0 + r, gk = k0 + c;
      xs[c][r] = (gs < S && gk < K) ? X[(size_t)gs * K + gk] : 0;
      int gn = n0 + r;
      int32_t wv = 0, uv = 0;
      if (gn < N && gk < K) {
        size_t off = (size_t)gn * K + gk;
        wv = w.width == 16 ? (int32_t) static_cast<const int16_t*>(w.p)[off] : static_cast<const int32_t*>(w.p)[off];
        if (PAIR) uv = wu.width == 16 ? (int32_t) static_cast<const int16_t*>(wu.p)[off] : static_cast<const int32_t*>(wu.p)[off];
      }
      ws[c][r] = wv;
      if (PAIR) us[c][r] = uv;
    }
    __syncthreads();
#pragma unroll 8
    for (int c = 0; c < LT_BK; ++c) {
      int32_t xv[4], wv[4], uv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) { xv[i] = xs[c][ty + 16 * i]; wv[i] = ws[c][tx + 16 * i]; }
      if (PAIR) {
#pragma unroll
        for (int i = 0; i < 4; ++i) uv[i] = us[c][tx + 16 * i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[i][j] = mac_wide(acc[i][j], xv[i], wv[j]);
          if (PAIR) accu[i][j] = mac_wide(accu[i][j], xv[i], uv[j]);
        }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int gs = s0 + ty + 16 * i, gn = n0 + tx + 16 * j;
      if (gs < S && gn < N) {
        int32_t v = requantize(acc[i][j]);
        if (PAIR) v = mul_sat(gelu_act(v), requantize(accu[i][j]));
        else if (epi == kEpiGeluMul) v = mul_sat(gelu_act(v), vec[(size_t)gs * N + gn]);
        Y[(size_t)gs * N + gn] = v;
      }
    }
}

void launch_linear(const int32_t* X, int32_t S, const DevMat& w, int32_t* Y, int32_t epi, const int32_t* vec,
                   cudaStream_t s) {
  dim3 grid((w.rows + LT_BN - 1) / LT_BN, (S + LT_BM - 1) / LT_BM);
  launch_k(linear_kernel<false>, dim3(grid), dim3(256), 0, s, X, S, w, w, Y, epi, vec);
}
void launch_linear_geglu(const int32_t* X, int32_t S, const DevMat& wg, const DevMat& wu, int32_t* Y,
                         cudaStream_t s) {
  dim3 grid((wg.rows + LT_BN - 1) / LT_BN, (S + LT_BM - 1) / LT_BM);
  launch_k(linear_kernel<true>, dim3(grid), dim3(256), 0, s, X, S, wg, wu, Y, kEpiPlain, nullptr);
}

// ---------------------------------------------------------------------------
// row norms
// ---------------------------------------------------------------------------
__global__ void rmsnorm_rows_kernel(const int32_t* x, int n, const int32_t* g, int64_t eps, int32_t* y) {
  pdl_entry();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int32_t* xs = reinterpret_cast<int32_t*>(smem_raw);
  __shared__ uint64_t red[33];
  const int32_t* xr = x + (size_t)blockIdx.x * n;
  for (int i = threadIdx.x; i < n; i += blockDim.x) xs[i] = xr[i];
  __syncthreads();
  int32_t sc = block_norm_scale(xs, n, eps, red);
  int32_t* yr = y + (size_t)blockIdx.x * n;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    int32_t v = mul_sat(xs[i], sc);
    yr[i] = g ? mul_sat(v, g[i]) : v;
  }
}
void launch_rmsnorm_rows(const int32_t* x, int32_t S, int32_t n, const int32_t* g, int64_t eps, int32_t* y,
                         cudaStream_t s) {
  size_t smem = (size_t)n * 4;
  if (smem > 48 * 1024) cudaFuncSetAttribute(rmsnorm_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  launch_k(rmsnorm_rows_kernel, dim3(S), dim3(256), smem, s, x, n, g, eps, y);
}

__global__ void norm_residual_kernel(const int32_t* a, const int32_t* res, int n, const int32_t* g, int64_t eps,
                                     bool has_scalar, int32_t scalar, int32_t* out) {
  pdl_entry();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int32_t* xs = reinterpret_cast<int32_t*>(smem_raw);
  __shared__ uint64_t red[33];
  size_t base = (size_t)blockIdx.x * n;
  for (int i = threadIdx.x; i < n; i += blockDim.x) xs[i] = a[base + i];
  __syncthreads();
  int32_t sc = block_norm_scale(xs, n, eps, red);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    int32_t t = add_sat(res[base + i], mul_sat(mul_sat(xs[i], sc), g[i]));
    if (has_scalar) t = mul_sat(t, scalar);
    out[base + i] = t;
  }
}
void launch_norm_residual_rows(const int32_t* a, const int32_t* res, int32_t S, int32_t n, const int32_t* g,
                               int64_t eps, bool has_scalar, int32_t scalar, int32_t* out, cudaStream_t s) {
  size_t smem = (size_t)n * 4;
  if (smem > 48 * 1024) cudaFuncSetAttribute(norm_residual_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  launch_k(norm_residual_kernel, dim3(S), dim3(256), smem, s, a, res, n, g, eps, has_scalar, scalar, out);
}

// Fused row norms (RowNormArgs in kernels.h).  One block per row, n % 4 == 0,
// every pointer 16-byte aligned (the launcher's caller checks).
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void row_norm_kernel(const RowNormArgs a, int S) {
  pdl_entry();
  if (a.wait_mask) {
    // the peers' sums of this reduction have been published
    if (threadIdx.x == 0) {
      for (int r = 0; r < 32; ++r) {
        if (!((a.wait_mask >> r) & 1u)) continue;
        uint32_t it = 0;
        while (ld_acquire_sys(a.flags + r) < a.wait_seq && ++it < (1u << 22)) __nanosleep(64);
        if (it >= (1u << 22)) atomicExch(&g_stream_err, 1);
      }
    }
    __syncthreads();
  }
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int4* xs = reinterpret_cast<int4*>(smem_raw);
  __shared__ uint64_t red[33];
  const int r = blockIdx.x, n = a.n, nq = n >> 2;
  const int4* ar = reinterpret_cast<const int4*>(a.a + (size_t)r * n);
  const longlong2* ar64 = reinterpret_cast<const longlong2*>(a.a64 + (size_t)r * n);
  uint64_t s = 0;
  for (int q = threadIdx.x; q < nq; q += blockDim.x) {
    int4 v;
    if (a.a64) {
      longlong2 x0 = ar64[2 * q], x1 = ar64[2 * q + 1];
      for (int i = 0; i < a.npeer; ++i) {  // wrapping i64 sums: order-free
        const longlong2* pr = reinterpret_cast<const longlong2*>(a.a64_peer[i] + (size_t)r * n);
        const longlong2 y0 = __ldcv(pr + 2 * q), y1 = __ldcv(pr + 2 * q + 1);
        x0.x = (long long)((unsigned long long)x0.x + (unsigned long long)y0.x);
        x0.y = (long long)((unsigned long long)x0.y + (unsigned long long)y0.y);
        x1.x = (long long)((unsigned long long)x1.x + (unsigned long long)y1.x);
        x1.y = (long long)((unsigned long long)x1.y + (unsigned long long)y1.y);
      }
      v = make_int4(requantize(x0.x), requantize(x0.y), requantize(x1.x), requantize(x1.y));
    } else {
      v = ar[q];
    }
    xs[q] = v;
    s = sat_add_u(s, (uint64_t)mul_wide(v.x, v.x));
    s = sat_add_u(s, (uint64_t)mul_wide(v.y, v.y));
    s = sat_add_u(s, (uint64_t)mul_wide(v.z, v.z));
    s = sat_add_u(s, (uint64_t)mul_wide(v.w, v.w));
  }
  const int32_t sc = block_norm_scale_partial(s, n, a.eps, red);
  const int4* g1 = reinterpret_cast<const int4*>(a.g1);
  auto nrm = [](int32_t x, int32_t k, int32_t g) { return mul_sat(mul_sat(x, k), g); };
  auto out_of24 = [](int4 y) {
    return y.x < -(1 << 23) || y.x >= (1 << 23) || y.y < -(1 << 23) || y.y >= (1 << 23) || y.z < -(1 << 23) ||
           y.z >= (1 << 23) || y.w < -(1 << 23) || y.w >= (1 << 23);
  };
  // the output row y is left in xs (and y_out); wide: some value needs 32 bits
  int wide = 0;
  auto keep = [&](int q, int4 y) {
    xs[q] = y;
    if (a.y_out) reinterpret_cast<int4*>(a.y_out + (size_t)r * n)[q] = y;
    wide |= out_of24(y);
  };
  if (a.res) {
    const int4* rr = reinterpret_cast<const int4*>(a.res + (size_t)r * n);
    uint64_t s2 = 0;
    for (int q = threadIdx.x; q < nq; q += blockDim.x) {
      const int4 x = xs[q], rv = rr[q], g = g1[q];
      int4 t = make_int4(add_sat(rv.x, nrm(x.x, sc, g.x)), add_sat(rv.y, nrm(x.y, sc, g.y)),
                         add_sat(rv.z, nrm(x.z, sc, g.z)), add_sat(rv.w, nrm(x.w, sc, g.w)));
      if (a.has_scalar)
        t = make_int4(mul_sat(t.x, a.scalar), mul_sat(t.y, a.scalar), mul_sat(t.z, a.scalar), mul_sat(t.w, a.scalar));
      xs[q] = t;
      if (a.t_out) reinterpret_cast<int4*>(a.t_out + (size_t)r * n)[q] = t;
      if (a.scatter) reinterpret_cast<int4*>(a.scatter[r] + a.scatter_off)[q] = t;
      s2 = sat_add_u(s2, (uint64_t)mul_wide(t.x, t.x));
      s2 = sat_add_u(s2, (uint64_t)mul_wide(t.y, t.y));
      s2 = sat_add_u(s2, (uint64_t)mul_wide(t.z, t.z));
      s2 = sat_add_u(s2, (uint64_t)mul_wide(t.w, t.w));
      if (!a.g2) wide |= out_of24(t);
    }
    if (a.g2) {
      const int32_t sc2 = block_norm_scale_partial(s2, n, a.eps, red);
      const int4* g2 = reinterpret_cast<const int4*>(a.g2);
      for (int q = threadIdx.x; q < nq; q += blockDim.x) {
        const int4 t = xs[q], g = g2[q];
        keep(q, make_int4(nrm(t.x, sc2, g.x), nrm(t.y, sc2, g.y), nrm(t.z, sc2, g.z), nrm(t.w, sc2, g.w)));
      }
    }
  } else {
    for (int q = threadIdx.x; q < nq; q += blockDim.x) {
      const int4 x = xs[q], g = g1[q];
      keep(q, make_int4(nrm(x.x, sc, g.x), nrm(x.y, sc, g.y), nrm(x.z, sc, g.z), nrm(x.w, sc, g.w)));
    }
  }
  if (!a.planes) return;
  // byte planes and row sum of y + 2^e: e = 23 when the whole row fits 24
  // bits (the row sum then carries the top-bit flag), else 31 (and the row's
  // 256-row tile is marked as needing the fourth limb)
  const bool four = __syncthreads_or(wide) != 0;
  const uint32_t off = four ? 0x80000000u : 0x00800000u;
  const size_t plane = (size_t)S * n;
  uint64_t usum = 0;
  for (int q = threadIdx.x; q < nq; q += blockDim.x) {
    const int4 y = xs[q];
    const uint32_t u[4] = {(uint32_t)y.x + off, (uint32_t)y.y + off, (uint32_t)y.z + off, (uint32_t)y.w + off};
    usum += (uint64_t)u[0] + u[1] + u[2] + u[3];
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const uint32_t packed = ((u[0] >> (8 * b)) & 0xffu) | (((u[1] >> (8 * b)) & 0xffu) << 8) |
                              (((u[2] >> (8 * b)) & 0xffu) << 16) | (((u[3] >> (8 * b)) & 0xffu) << 24);
      *reinterpret_cast<uint32_t*>(a.planes + b * plane + (size_t)r * n + 4 * q) = packed;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) usum += __shfl_xor_sync(0xffffffffu, usum, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = usum;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint64_t t = 0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
    a.rowsum[r] = four ? t : (t | (1ull << 63));
    if (four && a.tile4) atomicOr(&a.tile4[r / 256], 1u);
  }
}
void launch_row_norm(const RowNormArgs& a, int32_t rows, cudaStream_t s) {
  const size_t smem = (size_t)a.n * 4;
  if (smem > 48 * 1024) cudaFuncSetAttribute(row_norm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  // few rows (a batched decode step): one 16-byte piece per thread, so each
  // row's dependent norm phases run as short as they can; many rows
  // (prefill): 256 threads, several blocks per SM
  int threads = 256;
  if (rows < 2 * sm_count()) threads = std::max(256, std::min(1024, (a.n / 4 + 31) / 32 * 32));
  launch_k(row_norm_kernel, dim3(rows), dim3(threads), smem, s, a, (int)rows);
}

// ---------------------------------------------------------------------------
// q/k head norms, RoPE, value norm, KV-cache write.  One block per (row, head).
// ---------------------------------------------------------------------------
__device__ void rope_inplace(int32_t* v, int rotary, const int64_t* inv_freq, uint32_t pos) {
  if (rotary == 0 || pos == 0) return;
  int half = rotary >> 1;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    int32_t c, s;
    sin_cos_acc(pos_angle(pos, inv_freq[i]), &c, &s);
    int32_t l = v[i], r = v[i + half];
    v[i] = sub_sat(mul_sat(l, c), mul_sat(r, s));
    v[i + half] = add_sat(mul_sat(r, c), mul_sat(l, s));
  }
}

// rope_inplace with the (cos, sin) pairs of this position from a table
__device__ void rope_inplace_tab(int32_t* v, int rotary, const int32_t* cs, uint32_t pos) {
  if (rotary == 0 || pos == 0) return;
  int half = rotary >> 1;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const int2 t = reinterpret_cast<const int2*>(cs)[i];
    int32_t l = v[i], r = v[i + half];
    v[i] = sub_sat(mul_sat(l, t.x), mul_sat(r, t.y));
    v[i + half] = add_sat(mul_sat(r, t.x), mul_sat(l, t.y));
  }
}

__global__ void rope_table_kernel(const int64_t* inv_freq, int half, int32_t* cs) {
  pdl_entry();
  const uint32_t p = blockIdx.x;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    int32_t c, sn;
    sin_cos_acc(pos_angle(p, inv_freq[i]), &c, &sn);
    reinterpret_cast<int2*>(cs)[(size_t)p * half + i] = make_int2(c, sn);
  }
}
void launch_rope_table(const int64_t* inv_freq, int half, int S, int32_t* cs, cudaStream_t s) {
  launch_k(rope_table_kernel, dim3(S), dim3(half < 128 ? (half + 31) / 32 * 32 : 128), 0, s, inv_freq, half, cs);
}
// The same factors for batch row r at its own position *pos_rows[r].
__global__ void rope_rows_kernel(const int64_t* inv_freq, int half, const int32_t* const* pos_rows, int32_t* cs) {
  pdl_entry();
  const int r = blockIdx.x;
  const uint32_t p = (uint32_t)*pos_rows[r];
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    int32_t c, sn;
    sin_cos_acc(pos_angle(p, inv_freq[i]), &c, &sn);
    reinterpret_cast<int2*>(cs)[(size_t)r * half + i] = make_int2(c, sn);
  }
}
void launch_rope_rows(const int64_t* inv_freq, int half, int rows, const int32_t* const* pos_rows, int32_t* cs,
                      cudaStream_t s) {
  launch_k(rope_rows_kernel, dim3(rows), dim3(half < 128 ? (half + 31) / 32 * 32 : 128), 0, s, inv_freq, half,
           pos_rows, cs);
}

__global__ void qkv_post_kernel(const QkvPostArgs a) {
  pdl_entry();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int32_t* vs = reinterpret_cast<int32_t*>(smem_raw);
  __shared__ uint64_t red[33];
  const int s = blockIdx.x, head = blockIdx.y, d = a.d;
  const bool rows = a.pos_rows != nullptr;
  const uint32_t pos = rows ? (uint32_t)*a.pos_rows[s] : (uint32_t)(*a.pos + s);
  if (head < a.Hq) {
    const int32_t* src = a.q_in + (size_t)s * (a.ld ? a.ld : a.Hq * d) + (size_t)head * d;
    for (int i = threadIdx.x; i < d; i += blockDim.x) vs[i] = src[i];
    __syncthreads();
    int32_t sc = block_norm_scale(vs, d, a.eps, red);
    for (int i = threadIdx.x; i < d; i += blockDim.x) vs[i] = mul_sat(mul_sat(vs[i], sc), a.q_norm[i]);
    __syncthreads();
    if (a.rope_cs) rope_inplace_tab(vs, a.rotary, a.rope_cs + (size_t)s * a.rotary, pos);
    else rope_inplace(vs, a.rotary, a.inv_freq, pos);
    __syncthreads();
    int32_t* dst = a.q_out + ((size_t)s * a.Hq + head) * d;
    for (int i = threadIdx.x; i < d; i += blockDim.x) dst[i] = vs[i];
    return;
  }
  if (!a.k_in) return;
  // this layer appends K/V: the cache tables are set (a KV-sharing layer has none)
  int32_t* const kcache = rows ? a.kc_rows[s] : a.k_cache;
  int32_t* const vcache = rows ? a.vc_rows[s] : a.v_cache;
  const int cap = rows ? a.cap_rows[s] : a.cap;
  const int h = head - a.Hq;
  // K: head norm + RoPE
  const int32_t* ks = a.k_in + (size_t)s * (a.ld ? a.ld : a.Hkv * d) + (size_t)h * d;
  for (int i = threadIdx.x; i < d; i += blockDim.x) vs[i] = ks[i];
  __syncthreads();
  int32_t sc = block_norm_scale(vs, d, a.eps, red);
  for (int i = threadIdx.x; i < d; i += blockDim.x) vs[i] = mul_sat(mul_sat(vs[i], sc), a.k_norm[i]);
  __syncthreads();
  if (a.rope_cs) rope_inplace_tab(vs, a.rotary, a.rope_cs + (size_t)s * a.rotary, pos);
  else rope_inplace(vs, a.rotary, a.inv_freq, pos);
  __syncthreads();
  int32_t* kd = kcache + ((size_t)h * cap + pos) * d;
  for (int i = threadIdx.x; i < d; i += blockDim.x) kd[i] = vs[i];
  __syncthreads();
  // V: weightless value norm of the raw projection
  const int32_t* vsrc = a.v_in + (size_t)s * (a.ld ? a.ld : a.Hkv * d) + (size_t)h * d;
  for (int i = threadIdx.x; i < d; i += blockDim.x) vs[i] = vsrc[i];
  __syncthreads();
  int32_t sv = block_norm_scale(vs, d, a.eps, red);
  int32_t* vd = vcache + ((size_t)h * cap + pos) * d;
  for (int i = threadIdx.x; i < d; i += blockDim.x) vd[i] = mul_sat(vs[i], sv);
}
void launch_qkv_post(const QkvPostArgs& a, cudaStream_t s) {
  dim3 grid(a.S, a.Hq + (a.k_in ? a.Hkv : 0));
  launch_k(qkv_post_kernel, dim3(grid), dim3(128), (size_t)a.d * 4, s, a);
}

// ---------------------------------------------------------------------------
// decode attention: exact softmax in four grid-wide phases over splits of the
// key window (attention_output_into, det_kernels.rs:340-367).
// ---------------------------------------------------------------------------
// The attended rows [start, start + n) of batch row `row` (its position's
// window over its own cache).
__device__ __forceinline__ void decode_window(const AttnDecodeArgs& a, int row, int* start, int* n) {
  int len = (a.pos_rows ? *a.pos_rows[row] : (a.pos ? *a.pos : a.pos_value)) + 1;
  int st = (a.window > 0 && len > a.window) ? len - a.window : 0;
  *start = st;
  *n = len - st;
}

// phase 1: scores for the G query heads of one KV head over one split.
__global__ void attn_dec_scores(const AttnDecodeArgs a) {
  pdl_entry();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int32_t* qs = reinterpret_cast<int32_t*>(smem_raw);  // [G, d]
  __shared__ int32_t wmax[8][8];
  __shared__ int32_t widx[8][8];
  const int kvh = blockIdx.x, split = blockIdx.y, d = a.d;
  const int G = a.Hq / a.Hkv;
  int start, n;
  decode_window(a, (int)blockIdx.z, &start, &n);
  const int lo = split * a.rows_per_split, hi = min(n, lo + a.rows_per_split);
  for (int i = threadIdx.x; i < G * d; i += blockDim.x) qs[i] = a.q[(size_t)kvh * G * d + i];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarp = blockDim.x >> 5;
  int32_t bm[8];
  int32_t bi[8];
  for (int g = 0; g < G; ++g) { bm[g] = INT32_MIN; bi[g] = INT32_MAX; }
  for (int j = lo + warp; j < hi; j += nwarp) {
    const int32_t* kr = a.k_cache + ((size_t)kvh * a.cap + start + j) * d;
    int64_t acc[8];
    for (int g = 0; g < G; ++g) acc[g] = 0;
    for (int i = lane; i < d; i += 32) {
      int64_t kv = kr[i];
      for (int g = 0; g < G; ++g) acc[g] += kv * qs[g * d + i];
    }
    for (int g = 0; g < G; ++g) {
      int32_t sc = requantize(warp_sum64(acc[g]));
      if (lane == 0) a.sc.scores[(size_t)(kvh * G + g) * a.sc.stride + j] = sc;
      // j increases: the first max is kept (a row whose scores all equal
      // INT32_MIN takes its first row)
      if (sc > bm[g] || bi[g] == INT32_MAX) { bm[g] = sc; bi[g] = j; }
    }
  }
  if (lane == 0)
    for (int g = 0; g < G; ++g) { wmax[warp][g] = bm[g]; widx[warp][g] = bi[g]; }
  __syncthreads();
  if (threadIdx.x < G) {
    int g = threadIdx.x;
    int32_t m = INT32_MIN, mi = INT32_MAX;
    for (int w = 0; w < nwarp; ++w) {
      int32_t v = wmax[w][g], ix = widx[w][g];
      if (ix == INT32_MAX) continue;
      if (v > m || (v == m && ix < mi)) { m = v; mi = ix; }
    }
    size_t o = (size_t)(kvh * G + g) * a.sc.max_splits + split;
    a.sc.pmax[o] = m;
    a.sc.pidx[o] = mi;
  }
}

__device__ __forceinline__ void global_max(const AttnDecodeArgs& a, int h, int nsplit, int32_t* m, int32_t* mi) {
  int32_t bm = INT32_MIN, bi = INT32_MAX;
  for (int s = 0; s < nsplit; ++s) {
    size_t o = (size_t)h * a.sc.max_splits + s;
    int32_t v = a.sc.pmax[o], ix = a.sc.pidx[o];
    if (ix == INT32_MAX) continue;
    if (v > bm || (v == bm && ix < bi)) { bm = v; bi = ix; }
  }
  *m = bm;
  *mi = bi;
}

// phase 2: exp terms and partial sums
__global__ void attn_dec_exp(const AttnDecodeArgs a) {
  pdl_entry();
  __shared__ int32_t gmax[8];
  __shared__ uint64_t red[8][8];
  const int kvh = blockIdx.x, split = blockIdx.y;
  const int G = a.Hq / a.Hkv;
  int start, n;
  decode_window(a, (int)blockIdx.z, &start, &n);
  const int nsplit = (n + a.rows_per_split - 1) / a.rows_per_split;
  const int lo = split * a.rows_per_split, hi = min(n, lo + a.rows_per_split);
  if (threadIdx.x < G) {
    int32_t m, mi;
    global_max(a, kvh * G + threadIdx.x, nsplit, &m, &mi);
    gmax[threadIdx.x] = m;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarp = blockDim.x >> 5;
  for (int g = 0; g < G; ++g) {
    int h = kvh * G + g;
    uint64_t s = 0;
    for (int j = lo + threadIdx.x; j < hi; j += blockDim.x) {
      int64_t e = exp_term(a.sc.scores[(size_t)h * a.sc.stride + j], gmax[g]);
      a.sc.exps[(size_t)h * a.sc.stride + j] = e;
      s += (uint64_t)e;
    }
    s = (uint64_t)warp_sum64((int64_t)s);
    if (lane == 0) red[warp][g] = s;
  }
  __syncthreads();
  if (threadIdx.x < G) {
    uint64_t t = 0;
    for (int w = 0; w < nwarp; ++w) t += red[w][threadIdx.x];
    a.sc.psum[(size_t)(kvh * G + threadIdx.x) * a.sc.max_splits + split] = (int64_t)t;
  }
}

// phase 3: weights and partial weighted sums over V
__global__ void attn_dec_wsum(const AttnDecodeArgs a) {
  pdl_entry();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int32_t* ws = reinterpret_cast<int32_t*>(smem_raw);  // [G, rows_per_split]
  __shared__ int64_t tsum[8];
  __shared__ int64_t red[8][8];
  const int kvh = blockIdx.x, split = blockIdx.y, d = a.d;
  const int G = a.Hq / a.Hkv, R = a.rows_per_split;
  int start, n;
  decode_window(a, (int)blockIdx.z, &start, &n);
  const int nsplit = (n + R - 1) / R;
  const int lo = split * R, hi = min(n, lo + R);
  if (threadIdx.x < G) {
    int64_t t = 0;
    for (int s = 0; s < nsplit; ++s) t += a.sc.psum[(size_t)(kvh * G + threadIdx.x) * a.sc.max_splits + s];
    tsum[threadIdx.x] = t;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarp = blockDim.x >> 5;
  for (int g = 0; g < G; ++g) {
    int h = kvh * G + g;
    int64_t wsum = 0;
    for (int j = lo + threadIdx.x; j < lo + R; j += blockDim.x) {
      int32_t w = 0;
      if (j < hi) w = softmax_weight(a.sc.exps[(size_t)h * a.sc.stride + j], tsum[g]);
      ws[g * R + (j - lo)] = w;
      wsum += w;
    }
    wsum = warp_sum64(wsum);
    if (lane == 0) red[warp][g] = wsum;
  }
  __syncthreads();
  if (threadIdx.x < G) {
    int64_t t = 0;
    for (int w = 0; w < nwarp; ++w) t += red[w][threadIdx.x];
    a.sc.pwsum[(size_t)(kvh * G + threadIdx.x) * a.sc.max_splits + split] = t;
  }
  // partial weighted sum: thread per dim, loop over rows
  for (int dim = threadIdx.x; dim < d; dim += blockDim.x) {
    int64_t acc[8];
    for (int g = 0; g < G; ++g) acc[g] = 0;
    for (int j = lo; j < hi; ++j) {
      int64_t v = a.v_cache[((size_t)kvh * a.cap + start + j) * d + dim];
      for (int g = 0; g < G; ++g) acc[g] += v * ws[g * R + (j - lo)];
    }
    for (int g = 0; g < G; ++g) a.sc.pacc[((size_t)(kvh * G + g) * a.sc.max_splits + split) * d + dim] = acc[g];
  }
}

// phase 4: combine splits, residual to the first max, requantize.
__global__ void attn_dec_final(const AttnDecodeArgs a) {
  pdl_entry();
  const int h = blockIdx.x, d = a.d, G = a.Hq / a.Hkv, kvh = h / G;
  int start, n;
  decode_window(a, (int)blockIdx.z, &start, &n);
  const int nsplit = (n + a.rows_per_split - 1) / a.rows_per_split;
  __shared__ int32_t s_res, s_mi;
  if (threadIdx.x == 0) {
    int32_t m, mi;
    global_max(a, h, nsplit, &m, &mi);
    int64_t ws = 0;
    for (int s = 0; s < nsplit; ++s) ws += a.sc.pwsum[(size_t)h * a.sc.max_splits + s];
    int32_t wsum = ws > INT32_MAX ? INT32_MAX : (int32_t)ws;
    s_res = sub_sat(kOneAct, wsum);
    s_mi = mi;
  }
  __syncthreads();
  for (int dim = threadIdx.x; dim < d; dim += blockDim.x) {
    int64_t acc = 0;
    for (int s = 0; s < nsplit; ++s) acc += a.sc.pacc[((size_t)h * a.sc.max_splits + s) * d + dim];
    acc += (int64_t)a.v_cache[((size_t)kvh * a.cap + start + s_mi) * d + dim] * s_res;
    a.out[(size_t)h * d + dim] = requantize(acc);
  }
}

void launch_attn_decode(const AttnDecodeArgs& a, cudaStream_t s) {
  const int G = a.Hq / a.Hkv;
  dim3 grid(a.Hkv, a.sc.max_splits);
  launch_k(attn_dec_scores, dim3(grid), dim3(256), (size_t)G * a.d * 4, s, a);
  launch_k(attn_dec_exp, dim3(grid), dim3(256), 0, s, a);
  launch_k(attn_dec_wsum, dim3(grid), dim3(256), (size_t)G * a.rows_per_split * 4, s, a);
  launch_k(attn_dec_final, dim3(a.Hq), dim3(256), 0, s, a);
}

// ---------------------------------------------------------------------------
// decode attention, cluster version.  One thread-block cluster per group of
// GC query heads of one KV head; CTA r of the cluster takes rows
// [n*r/CL, n*(r+1)/CL) of the window.  GC is the smallest group that lets all
// clusters be resident at once (a 16-CTA cluster needs 16 SMs of one GPC).
// Exactly the arithmetic of attention_output_into: the first max, exp terms,
// sum and weights are cluster-wide values combined through distributed shared
// memory, and the weighted V sums (wrapping i64) are added across CTAs.
//
// Data path: model constants (norm gains, RoPE inverse frequencies) are
// requested before the grid-dependency wait; right after it thread 0 starts
// bulk copies (TMA, into this CTA's own shared memory) of its K rows and then V rows -- one
// contiguous span each -- into a ring of 32 KB shared-memory slots, each
// with an mbarrier that counts the bytes.  Waits are bounded: a wait that
// gives up sets the library's pipeline error flag (the host raises an error)
// instead of hanging.  With the fused prologue every CTA builds the current
// token's K/V row itself and reads it from shared memory, so clusters of one
// KV head never wait on each other; one CTA per KV head appends the row to
// the cache.  Cluster-wide reductions read one rank per lane and finish with
// warp shuffles.
// ---------------------------------------------------------------------------
namespace cg = cooperative_groups;
constexpr int kAcThreads = 256;
constexpr int kAcWarps = kAcThreads / 32;
constexpr int kAcTileBytes = 32 * 1024;
constexpr int kAcStages = 4;
constexpr int kAcVmx = 256;  // output dims one CTA finalises at most (first-max V row staging)

// acc + k . q over one 16-byte chunk (wrapping)
__device__ __forceinline__ int64_t dot4_acc(int64_t acc, const int4& k, const int4& q) {
  return mac_wide(mac_wide(mac_wide(mac_wide(acc, k.x, q.x), k.y, q.y), k.z, q.z), k.w, q.w);
}
__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(sa), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

struct AcLayout {  // offsets in 4-byte words of the dynamic shared memory
  int ring, qs, kvrow, qn, kn, ifq, sc, ex, pacc, total;
};
__host__ __device__ inline AcLayout ac_layout(int gc, int d, int rmax) {
  AcLayout L;
  int o = 0;
  L.ring = o; o += kAcStages * kAcTileBytes / 4;  // 16-byte aligned slots first
  L.qs = o; o += gc * d;
  L.kvrow = o; o += 2 * d;
  L.qn = o; o += d;
  L.kn = o; o += d;
  o = (o + 1) & ~1;
  L.ifq = o; o += 2 * 256;
  L.ex = o; o += 2 * gc * rmax;
  L.pacc = o; o += 2 * gc * d;
  L.sc = o; o += gc * rmax;
  L.total = o;
  return L;
}

// Sums each of the S per-lane values over the warp (S a power of two <= 32):
// transposed butterfly -- at each of the first log2(S) steps a lane keeps half
// of its values and trades the other half -- then plain xor steps.  Lane l
// returns the total of value l / (32 / S).  Wrapping i64 sums are order-free,
// so the result equals warp_sum64 of each value.
template <int S>
__device__ __forceinline__ int64_t warp_multi_sum(int64_t (&v)[S], int lane) {
#pragma unroll
  for (int cnt = S, o = 16; cnt > 1; cnt >>= 1, o >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < cnt / 2; ++i) {
      const int64_t send = up ? v[i] : v[i + cnt / 2];
      const int64_t keep = up ? v[i + cnt / 2] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  int64_t t = v[0];
#pragma unroll
  for (int o = 16 / S; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return t;
}

// (value, index) of the first maximum; index INT32_MAX marks "no rows"
__device__ __forceinline__ void first_max_merge(int32_t& v, int32_t& ix, int32_t ov, int32_t oi) {
  if (oi != INT32_MAX && (ix == INT32_MAX || ov > v || (ov == v && oi < ix))) { v = ov; ix = oi; }
}

// Head dims up to 128*NCH with d % 4 == 0; lane l owns 16-byte chunks
// l + 32u (u < NCH) of every row.
template <int GC, int NCH>
__global__ void __launch_bounds__(kAcThreads, 1) attn_dec_cluster_kernel(const AttnDecodeArgs a, int rmax) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int32_t* sm = reinterpret_cast<int32_t*>(smem_raw);
  cg::cluster_group cl = cg::this_cluster();
  const int CL = (int)cl.num_blocks(), rank = (int)cl.block_rank();
  const int d = a.d, nch = d >> 2;
  const int G = a.group ? a.group : a.Hq / a.Hkv;
  const int qh0 = blockIdx.y * GC;  // first (local) query head of this cluster
  const int kvh = (a.head0 + qh0) / G;
  const AcLayout Ly = ac_layout(GC, d, rmax);
  unsigned char* ring = smem_raw + (size_t)Ly.ring * 4;
  int32_t* qs = sm + Ly.qs;        // [GC][d]
  int32_t* kvrow = sm + Ly.kvrow;  // current token's k, v
  int32_t* qn = sm + Ly.qn;
  int32_t* kn = sm + Ly.kn;
  int64_t* ifq = reinterpret_cast<int64_t*>(sm + Ly.ifq);
  int32_t* sc = sm + Ly.sc;                                  // [GC][rmax] scores, then weights
  int64_t* ex = reinterpret_cast<int64_t*>(sm + Ly.ex);      // [GC][rmax]
  int64_t* pacc = reinterpret_cast<int64_t*>(sm + Ly.pacc);  // [GC][d]
  __shared__ __align__(8) uint64_t full[kAcStages];
  __shared__ int32_t s_max[GC], s_idx[GC], g_max[GC], g_idx[GC], g_res[GC], sc_q[GC], sc_kv[2];
  __shared__ int64_t s_sum[GC], s_wsum[GC], g_sum[GC];
  __shared__ int32_t wm[kAcWarps][GC], wi[kAcWarps][GC];
  __shared__ int64_t ws[kAcWarps][GC];
  __shared__ int32_t cs_tab[256], sn_tab[256];
  __shared__ int32_t vmx[GC][kAcVmx];  // first-max V row, this CTA's output dims
  __shared__ int s_fail;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const AttnFuse& f = a.fuse;
  const bool fused = f.q_in != nullptr;
  const bool new_row = fused && f.k_in != nullptr;  // this layer appends the current token
  const int half = fused ? (f.rotary >> 1) : 0;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // model constants, requested before the grid-dependency wait
  if (fused) {
    for (int i = tid; i < d; i += kAcThreads) {
      cp_async4(qn + i, f.q_norm + i);
      if (new_row) cp_async4(kn + i, f.k_norm + i);
    }
    for (int i = tid; i < half; i += kAcThreads) cp_async8(ifq + i, f.inv_freq + i);
  }
  if (tid == 0) {
    for (int i = 0; i < kAcStages; ++i) mbar_init(&full[i], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_fail = 0;
  }
  __syncthreads();
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // batched decode: cluster row blockIdx.z is its own sequence
  const int brow = a.row_order ? a.row_order[blockIdx.z] : (int)blockIdx.z;
  const bool batched = a.pos_rows != nullptr;
  const int32_t* const kc = batched ? a.kc_rows[brow] : a.k_cache;
  const int32_t* const vc = batched ? a.vc_rows[brow] : a.v_cache;
  const int capr = batched ? a.cap_rows[brow] : a.cap;
  const int32_t* const qrow = a.q + (size_t)brow * a.Hq * d;
  int32_t* const orow = a.out + (size_t)brow * a.Hq * d;
  const int pos = batched ? *a.pos_rows[brow] : (a.pos ? *a.pos : a.pos_value);
  int start, n;
  decode_window(a, brow, &start, &n);
  const int lo = (int)((int64_t)n * rank / CL), hi = (int)((int64_t)n * (rank + 1) / CL);
  const int rows = hi - lo;
  const int TR = kAcTileBytes / (d * 4);  // rows per tile
  const int tiles = (rows + TR - 1) / TR;
  const int total_tiles = 2 * tiles;  // K tiles, then V tiles
  const size_t head_base = (size_t)kvh * capr;
  // the current token's row (when built here) is the CTA's last row and is
  // not copied from the cache
  const int copy_rows = rows - ((new_row && rows > 0 && start + hi - 1 == pos) ? 1 : 0);
  // unified tile u: K tile u (u < tiles) or V tile u - tiles, in slot u % S
  auto issue = [&](int u) {  // thread 0 only
    const int slot = u % kAcStages;
    const int t = u < tiles ? u : u - tiles;
    const int32_t* cache = u < tiles ? kc : vc;
    const int r0 = t * TR;
    const int nr = min(TR, copy_rows - r0);
    if (nr > 0) {
      const uint32_t bytes = (uint32_t)nr * d * 4;
      mbar_arrive_tx(&full[slot], bytes);
      bulk_g2s(ring + (size_t)slot * kAcTileBytes, cache + (head_base + start + lo + r0) * d, bytes, &full[slot]);
    } else {
      mbar_arrive(&full[slot]);
    }
  };
  auto wait_tile = [&](int u) {  // every thread
    if (!mbar_wait(&full[u % kAcStages], (u / kAcStages) & 1)) s_fail = 1;
  };
  if (tid == 0)
    for (int u = 0; u < kAcStages && u < total_tiles; ++u) issue(u);
  for (int i = tid; i < GC * d; i += kAcThreads) pacc[i] = 0;
  if (!fused) {
    for (int i = tid; i < GC * d; i += kAcThreads) qs[i] = qrow[(size_t)qh0 * d + i];
  } else {
    for (int i = tid; i < GC * d; i += kAcThreads) qs[i] = f.q_in[(size_t)qh0 * d + i];
    if (new_row)
      for (int i = tid; i < d; i += kAcThreads) {
        kvrow[i] = f.k_in[(size_t)kvh * d + i];
        kvrow[d + i] = f.v_in[(size_t)kvh * d + i];
      }
    cp_async_commit_wait_all();  // the constants have landed
    __syncthreads();
    for (int i = tid; i < half; i += kAcThreads) {
      int32_t cv, sv;
      sin_cos_acc(pos_angle((uint32_t)pos, ifq[i]), &cv, &sv);
      cs_tab[i] = cv;
      sn_tab[i] = sv;
    }
    if (warp >= kAcWarps - GC) {
      const int g = warp - (kAcWarps - GC);
      int32_t scv = warp_norm_scale(qs + g * d, d, f.eps);
      if (lane == 0) sc_q[g] = scv;
    } else if (new_row && warp == kAcWarps - GC - 1) {
      int32_t scv = warp_norm_scale(kvrow, d, f.eps);
      if (lane == 0) sc_kv[0] = scv;
    } else if (new_row && warp == kAcWarps - GC - 2) {
      int32_t scv = warp_norm_scale(kvrow + d, d, f.eps);
      if (lane == 0) sc_kv[1] = scv;
    }
    __syncthreads();
    for (int i = tid; i < GC * d; i += kAcThreads) {
      const int g = i / d, t = i - g * d;
      qs[i] = mul_sat(mul_sat(qs[i], sc_q[g]), qn[t]);
    }
    if (new_row)
      for (int i = tid; i < d; i += kAcThreads) {
        kvrow[i] = mul_sat(mul_sat(kvrow[i], sc_kv[0]), kn[i]);
        kvrow[d + i] = mul_sat(kvrow[d + i], sc_kv[1]);
      }
    __syncthreads();
    if (pos != 0 && half > 0) {  // rope_rotate_pairs_in_place leaves position 0 unchanged
      const int nv = GC + (new_row ? 1 : 0);
      for (int e = tid; e < nv * half; e += kAcThreads) {
        const int h = e / half, i = e - h * half;
        int32_t* v = h < GC ? qs + h * d : kvrow;
        const int32_t l = v[i], r = v[i + half];
        v[i] = sub_sat(mul_sat(l, cs_tab[i]), mul_sat(r, sn_tab[i]));
        v[i + half] = add_sat(mul_sat(r, cs_tab[i]), mul_sat(l, sn_tab[i]));
      }
    }
    if (new_row && rank == 0 && (a.head0 + qh0) % G == 0) {
      __syncthreads();
      for (int i = tid; i < d; i += kAcThreads) {
        f.k_out[(head_base + pos) * d + i] = kvrow[i];
        f.v_out[(head_base + pos) * d + i] = kvrow[d + i];
      }
    }
  }
  __syncthreads();
  // ---- phase 1: scores, tile by tile from shared memory.  A warp takes RB
  // rows at a time; the RB*GC dot products of a step are reduced together and
  // lane l owns value l / (32/S) (row l/(32/S)/GC of the step, head % GC).
  constexpr int RB = NCH >= 4 ? 2 : (NCH == 2 ? 4 : 8);
  constexpr int S = RB * GC;
  int4 qv[GC][NCH];
#pragma unroll
  for (int g = 0; g < GC; ++g)
#pragma unroll
    for (int u = 0; u < NCH; ++u) {
      const int c = lane + 32 * u;
      qv[g][u] = c < nch ? reinterpret_cast<const int4*>(qs + g * d)[c] : make_int4(0, 0, 0, 0);
    }
  const int own = lane / (32 / S);  // value index this lane finalizes
  const int own_r = own / GC, own_g = own % GC;
  const bool owner = lane % (32 / S) == 0;
  int32_t bm = INT32_MIN, bi = INT32_MAX;  // this lane's candidate for head own_g
  for (int t = 0; t < tiles; ++t) {
    wait_tile(t);
    const int r0 = t * TR, nr = min(TR, rows - r0);
    const int32_t* tile = reinterpret_cast<const int32_t*>(ring + (size_t)(t % kAcStages) * kAcTileBytes);
    for (int base = warp * RB; base < nr; base += kAcWarps * RB) {
      int64_t acc[S];
#pragma unroll
      for (int r = 0; r < RB; ++r) {
        const int i = base + r;
        int4 kv[NCH];
        const int4* kr = reinterpret_cast<const int4*>(
            (new_row && start + lo + r0 + i == pos) ? kvrow : tile + (size_t)(i < nr ? i : 0) * d);
#pragma unroll
        for (int u = 0; u < NCH; ++u) {
          const int c = lane + 32 * u;
          kv[u] = (i < nr && c < nch) ? kr[c] : make_int4(0, 0, 0, 0);
        }
#pragma unroll
        for (int g = 0; g < GC; ++g) {
          int64_t x = 0;
#pragma unroll
          for (int u = 0; u < NCH; ++u) x = dot4_acc(x, kv[u], qv[g][u]);
          acc[r * GC + g] = x;
        }
      }
      const int64_t tot = warp_multi_sum<S>(acc, lane);
      const int i = base + own_r;
      if (owner && i < nr) {
        const int j = r0 + i;
        const int32_t v = requantize(tot);
        sc[own_g * rmax + j] = v;
        if (v > bm || bi == INT32_MAX) { bm = v; bi = lo + j; }  // a lane's rows ascend: the first max is kept
      }
    }
    __syncthreads();
    if (tid == 0 && t + kAcStages < total_tiles) issue(t + kAcStages);
  }
  // per-head first max over the lanes that own the head, then over warps
#pragma unroll
  for (int g = 0; g < GC; ++g) {
    int32_t m = own_g == g ? bm : INT32_MIN, mi = own_g == g ? bi : INT32_MAX;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const int32_t om = __shfl_xor_sync(0xffffffffu, m, o), oi = __shfl_xor_sync(0xffffffffu, mi, o);
      first_max_merge(m, mi, om, oi);
    }
    if (lane == 0) { wm[warp][g] = m; wi[warp][g] = mi; }
  }
  __syncthreads();
  if (tid < GC) {
    const int g = tid;
    int32_t m = INT32_MIN, mi = INT32_MAX;
    for (int w = 0; w < kAcWarps; ++w) first_max_merge(m, mi, wm[w][g], wi[w][g]);
    s_max[g] = m;
    s_idx[g] = mi;
  }
  cl.sync();
  // ---- global first max: warp g reads rank `lane` and reduces by shuffles
  if (warp < GC) {
    const int g = warp;
    int32_t m = INT32_MIN, mi = INT32_MAX;
    if (lane < CL) {
      m = *cl.map_shared_rank(&s_max[g], lane);
      mi = *cl.map_shared_rank(&s_idx[g], lane);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const int32_t om = __shfl_xor_sync(0xffffffffu, m, o), oi = __shfl_xor_sync(0xffffffffu, mi, o);
      first_max_merge(m, mi, om, oi);
    }
    if (lane == 0) { g_max[g] = m; g_idx[g] = mi; }
  }
  __syncthreads();
  // the combine's residual row v[first max], this CTA's dims, fetched early
  const int d0 = (int)((int64_t)d * rank / CL), d1 = (int)((int64_t)d * (rank + 1) / CL);
  const int per = d1 - d0;
  for (int e = tid; e < GC * per; e += kAcThreads) {
    const int g = e / per, dim = d0 + e % per;
    const int r = start + g_idx[g];
    if (new_row && r == pos) vmx[g][e % per] = kvrow[d + dim];
    else cp_async4(&vmx[g][e % per], vc + (head_base + r) * d + dim);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  // ---- phase 2: exp terms and local sums, (head, row) pairs in parallel
  {
    int64_t sum[GC];
#pragma unroll
    for (int g = 0; g < GC; ++g) sum[g] = 0;
    for (int e = tid; e < GC * rows; e += kAcThreads) {
      const int g = e / rows, j = e - g * rows;
      const int64_t x = exp_term(sc[g * rmax + j], g_max[g]);
      ex[g * rmax + j] = x;
#pragma unroll
      for (int h = 0; h < GC; ++h) sum[h] += h == g ? x : 0;
    }
    const int64_t t = warp_multi_sum<GC>(sum, lane);
    if (lane % (32 / GC) == 0) ws[warp][lane / (32 / GC)] = t;
  }
  __syncthreads();
  if (tid < GC) {
    int64_t t = 0;
    for (int w = 0; w < kAcWarps; ++w) t += ws[w][tid];
    s_sum[tid] = t;
  }
  cl.sync();
  if (warp < GC) {
    const int64_t v = lane < CL ? *cl.map_shared_rank(&s_sum[warp], lane) : 0;
    const int64_t t = warp_sum64(v);
    if (lane == 0) g_sum[warp] = t;
  }
  __syncthreads();
  // ---- phase 3: weights, local weight sums, partial weighted V sums
  {
    int64_t wsum[GC];
#pragma unroll
    for (int g = 0; g < GC; ++g) wsum[g] = 0;
    for (int e = tid; e < GC * rows; e += kAcThreads) {
      const int g = e / rows, j = e - g * rows;
      const int32_t w = softmax_weight(ex[g * rmax + j], g_sum[g]);
      sc[g * rmax + j] = w;
#pragma unroll
      for (int h = 0; h < GC; ++h) wsum[h] += h == g ? w : 0;
    }
    const int64_t t = warp_multi_sum<GC>(wsum, lane);
    if (lane % (32 / GC) == 0) ws[warp][lane / (32 / GC)] = t;
  }
  __syncthreads();
  if (tid < GC) {
    int64_t t = 0;
    for (int w = 0; w < kAcWarps; ++w) t += ws[w][tid];
    s_wsum[tid] = t;
  }
  int64_t acc[GC][NCH][4];
#pragma unroll
  for (int g = 0; g < GC; ++g)
#pragma unroll
    for (int u = 0; u < NCH; ++u)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[g][u][e] = 0;
  for (int t = 0; t < tiles; ++t) {
    const int uu = tiles + t;
    wait_tile(uu);
    const int r0 = t * TR, nr = min(TR, rows - r0);
    const int32_t* tile = reinterpret_cast<const int32_t*>(ring + (size_t)(uu % kAcStages) * kAcTileBytes);
    // two rows per warp step: both rows' V chunks and weights are loaded
    // before any multiply-add (rows past the tile load as zero weight x 0)
    for (int i0 = warp; i0 < nr; i0 += 2 * kAcWarps) {
      int4 vv[2][NCH];
      int32_t ww[2][GC];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int i = i0 + h * kAcWarps;
        const bool ok = i < nr;
        const int j = r0 + (ok ? i : 0);
        const int4* vr = reinterpret_cast<const int4*>(
            (new_row && start + lo + j == pos) ? kvrow + d : tile + (size_t)(ok ? i : 0) * d);
#pragma unroll
        for (int u = 0; u < NCH; ++u) {
          const int c = lane + 32 * u;
          vv[h][u] = (ok && c < nch) ? vr[c] : make_int4(0, 0, 0, 0);
        }
#pragma unroll
        for (int g = 0; g < GC; ++g) ww[h][g] = ok ? sc[g * rmax + j] : 0;
      }
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int u = 0; u < NCH; ++u)
#pragma unroll
          for (int g = 0; g < GC; ++g) {
            const int32_t w = ww[h][g];
            const int4 v = vv[h][u];
            acc[g][u][0] = mac_wide(acc[g][u][0], v.x, w);
            acc[g][u][1] = mac_wide(acc[g][u][1], v.y, w);
            acc[g][u][2] = mac_wide(acc[g][u][2], v.z, w);
            acc[g][u][3] = mac_wide(acc[g][u][3], v.w, w);
          }
    }
    __syncthreads();
    if (tid == 0 && uu + kAcStages < total_tiles) issue(uu + kAcStages);
  }
#pragma unroll
  for (int g = 0; g < GC; ++g)
#pragma unroll
    for (int u = 0; u < NCH; ++u) {
      const int c = lane + 32 * u;
      if (c < nch)
#pragma unroll
        for (int e = 0; e < 4; ++e)
          atomicAdd(reinterpret_cast<unsigned long long*>(&pacc[g * d + 4 * c + e]), (unsigned long long)acc[g][u][e]);
    }
  cl.sync();
  // ---- combine: this CTA finalizes output dims [d*rank/CL, d*(rank+1)/CL);
  // CL consecutive lanes read one element's partial sums from the CL ranks
  if (warp < GC) {
    const int64_t v = lane < CL ? *cl.map_shared_rank(&s_wsum[warp], lane) : 0;
    const int64_t t = warp_sum64(v);
    if (lane == 0) g_res[warp] = sub_sat(kOneAct, t > INT32_MAX ? INT32_MAX : (int32_t)t);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  const int nel = GC * per, epw = kAcThreads / CL;
  for (int base = 0; base < nel; base += epw) {
    const int e = base + tid / CL, r = tid % CL;
    int64_t v = 0;
    int g = 0, dim = 0;
    if (e < nel) {
      g = e / per;
      dim = d0 + e % per;
      v = *cl.map_shared_rank(&pacc[g * d + dim], r);
    }
    for (int o = CL >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (r == 0 && e < nel) {
      v += (int64_t)vmx[g][dim - d0] * g_res[g];
      orow[(size_t)(qh0 + g) * d + dim] = requantize(v);
    }
  }
  if (s_fail && tid == 0) {
    atomicExch(&g_stream_err, 1);
    // every issued copy has a consumer wait; give stragglers one more bounded
    // wait before the CTA's shared memory is released
    for (int u = max(0, total_tiles - kAcStages); u < total_tiles; ++u)
      mbar_wait(&full[u % kAcStages], (u / kAcStages) & 1);
  }
  cl.sync();  // keep this CTA's shared memory alive until every rank has read it
}

static int g_attn_cluster = 0;   // cluster size chosen for this device
static int g_attn_max_clusters = 0;  // 16- or 8-CTA clusters resident at once

static size_t ac_smem(int gc, int d, int rmax) { return (size_t)ac_layout(gc, d, rmax).total * 4; }

template <int GC, int NCH>
static cudaError_t launch_ac(const AttnDecodeArgs& a, int CL, int rmax, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(CL, a.Hq / GC, a.batch > 0 ? a.batch : 1);
  cfg.blockDim = dim3(kAcThreads, 1, 1);
  cfg.dynamicSmemBytes = ac_smem(GC, a.d, rmax);
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
  return cudaLaunchKernelEx(&cfg, attn_dec_cluster_kernel<GC, NCH>, a, rmax);
}

// dynamic shared memory cap: 227 KB per block minus the kernel's static
// shared memory (under 7 KB)
constexpr size_t kAcMaxSmem = 219 * 1024;

template <int GC, int NCH>
static void ac_prepare1(int CL) {
  cudaFuncSetAttribute(attn_dec_cluster_kernel<GC, NCH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kAcMaxSmem);
  if (CL > 8)
    cudaFuncSetAttribute(attn_dec_cluster_kernel<GC, NCH>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
}
template <int NCH>
static void ac_prepare(int CL) {
  ac_prepare1<1, NCH>(CL);
  ac_prepare1<2, NCH>(CL);
  ac_prepare1<4, NCH>(CL);
}

static int ac_max_clusters(int CL) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(CL, 1, 1);
  cfg.blockDim = dim3(kAcThreads, 1, 1);
  cfg.dynamicSmemBytes = ac_smem(1, 512, 300);  // one CTA per SM
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, attn_dec_cluster_kernel<1, 4>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  return n;
}

static void attn_cluster_init() {
  ac_prepare<1>(16);
  ac_prepare<2>(16);
  ac_prepare<4>(16);
  if (g_attn_cluster) return;
  // 16-CTA clusters when the device can schedule them, else the portable 8
  int n = ac_max_clusters(16);
  if (n >= 1) {
    g_attn_cluster = 16;
  } else {
    g_attn_cluster = 8;
    n = ac_max_clusters(8);
  }
  g_attn_max_clusters = n > 0 ? n : 1;
}

static int ac_rmax(int window, int cap, int CL) {
  const int span = window > 0 && window < cap ? window : cap;
  return (span + CL - 1) / CL + 1;
}

// Query heads per cluster: the smallest power of two dividing the group size
// G that keeps Hq/GC clusters resident together (capped by register budget).
static int ac_group(int Hq, int Hkv, int d) {
  const int G = Hq / Hkv;
  const int cap = d <= 256 ? 4 : 2;
  const int maxc = g_attn_max_clusters > 0 ? g_attn_max_clusters : 1;
  int gc = 1;
  while (Hq / gc > maxc && gc * 2 <= cap && G % (gc * 2) == 0) gc *= 2;
  return gc;
}

bool attn_decode_cluster_fits(int Hq, int Hkv, int d, int window, int cap, int rotary, int group) {
  const int CL = g_attn_cluster ? g_attn_cluster : 8;
  if (group == 0) {
    if (!(Hkv > 0 && Hq % Hkv == 0)) return false;
    group = Hq / Hkv;
  }
  if (!(d > 0 && d % 4 == 0 && d <= 512 && (rotary >> 1) <= 256)) return false;
  const int gl = std::max(1, std::min(group, Hq));
  if (Hq % gl != 0) return false;
  const int gc = ac_group(Hq, Hq / gl, d);
  return gc <= 8 - 2 && d <= kAcVmx * CL && ac_smem(gc, d, ac_rmax(window, cap, CL)) <= kAcMaxSmem;
}

// Cluster size of batched launches: the batch rows already fill the GPU, so
// each sequence gets a small cluster (fewer fixed per-CTA phase latencies).
#ifndef RDET_AC_BATCH_CL
#define RDET_AC_BATCH_CL 2
#endif

void launch_attn_decode_cluster(const AttnDecodeArgs& a, cudaStream_t s) {
  int CL = g_attn_cluster ? g_attn_cluster : 8;
  // batched, 512-dim heads: clusters of 8 so that all four query heads of a
  // KV head fit one cluster (K/V read once); else the smallest cluster
  const int Gq = a.group ? a.group : a.Hq / a.Hkv;
  const bool wide4 = a.batch > 1 && a.d > 256 && Gq % 4 == 0 && CL >= 8 &&
                     ac_smem(4, a.d, ac_rmax(a.window, a.cap, 8)) <= kAcMaxSmem && a.d <= kAcVmx * 8;
  if (a.batch > 1 && launch_attn_decode_tc(a, sm_count(), s)) return;
  if (a.batch > 1) {
    // a CTA finalises d / CL output dims (at most kAcVmx: the first-max V
    // row is staged in a [GC][kAcVmx] shared array).  One CTA per
    // (sequence, query group) when those CTAs fit one wave: a second,
    // partly filled wave of half-size CTAs costs more than longer CTAs.
    // With few query heads per GPU (tensor-parallel ranks) the one-CTA shape
    // leaves SMs idle: split each window over the largest cluster that
    // still fits one wave.
    const int groups = std::max(1, a.Hq / std::max(1, std::min(4, Gq)));
    const long ctas = (long)a.batch * groups;
    int one_wave = 1;
    while (one_wave < 4 && ctas * one_wave * 2 <= sm_count()) one_wave *= 2;
    int cl = wide4 ? (ac_smem(4, a.d, ac_rmax(a.window, a.cap, 4)) <= kAcMaxSmem ? 4 : 8)
                   : (ctas <= sm_count() ? one_wave : RDET_AC_BATCH_CL);
    while (cl < CL && (a.d > kAcVmx * cl || ac_smem(1, a.d, ac_rmax(a.window, a.cap, cl)) > kAcMaxSmem)) cl *= 2;
    CL = cl < CL ? cl : CL;
  }
  const int rmax = ac_rmax(a.window, a.cap, CL);
  // (batched rows use the library's own 16-byte aligned cache allocations)
  const bool aligned = ((reinterpret_cast<uintptr_t>(a.k_cache) | reinterpret_cast<uintptr_t>(a.v_cache)) & 15) == 0;
  if (!aligned ||
      !attn_decode_cluster_fits(a.Hq, a.Hkv, a.d, a.window, a.cap, a.fuse.q_in ? a.fuse.rotary : 0, a.group)) {
    launch_attn_decode(a, s);  // callers only fuse when the cluster kernel fits
    return;
  }
  // a cluster's GC query heads share one KV head: GC divides the model's group
  // size and the local head count
  const int G = a.group ? a.group : a.Hq / a.Hkv;
  const int Gl = std::min(G, a.Hq);
  int gc = ac_group(a.Hq, a.Hq / Gl, a.d);
  if (a.batch > 1) {  // many clusters already: share K/V reads between query heads
    const int cap = (a.d <= 256 || wide4) ? 4 : 2;
    while (gc * 2 <= cap && Gl % (gc * 2) == 0 && ac_smem(gc * 2, a.d, rmax) <= kAcMaxSmem) gc *= 2;
  }
  // launch errors surface through cudaGetLastError in the caller
  if (a.d <= 128) {
    if (gc == 1) launch_ac<1, 1>(a, CL, rmax, s);
    else if (gc == 2) launch_ac<2, 1>(a, CL, rmax, s);
    else launch_ac<4, 1>(a, CL, rmax, s);
  } else if (a.d <= 256) {
    if (gc == 1) launch_ac<1, 2>(a, CL, rmax, s);
    else if (gc == 2) launch_ac<2, 2>(a, CL, rmax, s);
    else launch_ac<4, 2>(a, CL, rmax, s);
  } else {
    if (gc == 1) launch_ac<1, 4>(a, CL, rmax, s);
    else if (gc == 2) launch_ac<2, 4>(a, CL, rmax, s);
    else launch_ac<4, 4>(a, CL, rmax, s);
  }
}

// ---------------------------------------------------------------------------
// prefill attention (causal + optional sliding window), one block per
// (head, query).  Scores live in global scratch rows of length `rowlen`.
// ---------------------------------------------------------------------------
__global__ void attn_prefill_kernel(const AttnPrefillArgs a, int rowlen) {
  pdl_entry();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int32_t* qs = reinterpret_cast<int32_t*>(smem_raw);
  __shared__ int32_t wm[32], wi[32];
  __shared__ uint64_t wr[32];
  __shared__ int32_t s_max, s_mi, s_res;
  __shared__ int64_t s_sum;
  const int h = blockIdx.x, i = blockIdx.y, d = a.d;
  const int G = a.Hq / a.Hkv, kvh = h / G;
  const int start = (a.window > 0 && i + 1 > a.window) ? i + 1 - a.window : 0;
  const int n = i + 1 - start;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarp = blockDim.x >> 5;
  for (int t = threadIdx.x; t < d; t += blockDim.x) qs[t] = a.q[((size_t)i * a.Hq + h) * d + t];
  __syncthreads();
  int32_t* sc = a.scores + ((size_t)h * a.S + i) * rowlen;
  int64_t* ex = a.exps + ((size_t)h * a.S + i) * rowlen;
  // scores + first max
  int32_t bm = INT32_MIN, bi = INT32_MAX;
  for (int j = warp; j < n; j += nwarp) {
    const int32_t* kr = a.k_cache + ((size_t)kvh * a.cap + start + j) * d;
    int64_t acc = 0;
    for (int t = lane; t < d; t += 32) acc = mac_wide(acc, kr[t], qs[t]);
    int32_t v = requantize(warp_sum64(acc));
    if (lane == 0) sc[j] = v;
    if (v > bm || bi == INT32_MAX) { bm = v; bi = j; }
  }
  if (lane == 0) { wm[warp] = bm; wi[warp] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    int32_t m = INT32_MIN, mi = INT32_MAX;
    for (int w = 0; w < nwarp; ++w) {
      if (wi[w] == INT32_MAX) continue;
      if (wm[w] > m || (wm[w] == m && wi[w] < mi)) { m = wm[w]; mi = wi[w]; }
    }
    s_max = m;
    s_mi = mi;
  }
  __syncthreads();
  // exp terms + sum
  uint64_t sum = 0;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    int64_t e = exp_term(sc[j], s_max);
    ex[j] = e;
    sum += (uint64_t)e;
  }
  sum = (uint64_t)warp_sum64((int64_t)sum);
  if (lane == 0) wr[warp] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint64_t t = 0;
    for (int w = 0; w < nwarp; ++w) t += wr[w];
    s_sum = (int64_t)t;
  }
  __syncthreads();
  // weights (stored over the scores) + weight sum
  int64_t wsum = 0;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    int32_t w = softmax_weight(ex[j], s_sum);
    sc[j] = w;
    wsum += w;
  }
  wsum = warp_sum64(wsum);
  if (lane == 0) wr[warp] = (uint64_t)wsum;
  __syncthreads();
  if (threadIdx.x == 0) {
    int64_t t = 0;
    for (int w = 0; w < nwarp; ++w) t += (int64_t)wr[w];
    s_res = sub_sat(kOneAct, t > INT32_MAX ? INT32_MAX : (int32_t)t);
    sc[s_mi] = add_sat(sc[s_mi], s_res);
  }
  __syncthreads();
  for (int t = threadIdx.x; t < d; t += blockDim.x) {
    int64_t acc = 0;
    const int32_t* vb = a.v_cache + ((size_t)kvh * a.cap + start) * d + t;
    for (int j = 0; j < n; ++j) acc = mac_wide(acc, vb[(size_t)j * d], sc[j]);
    a.out[((size_t)i * a.Hq + h) * d + t] = requantize(acc);
  }
}
// Tiled prefill attention: one CTA per (KV head, block of QB queries) covering
// all G query heads of the group (R = QB*G <= 64 query rows), with K and V
// streamed through shared memory in tiles of 32 keys.  Phase A writes exact
// scores to scratch and tracks the first max per row; phase B turns each row
// into exact softmax weights (exp, saturating-free sum, ties-to-even division,
// residual to the first max); phase C accumulates the weighted V sum in i64.
constexpr int AP_R = 64, AP_TK = 32, AP_CH = 128;
// RPW rows per warp: 8 warps of 8 rows when two CTAs share an SM (head_dim
// 256, ~106 KB each), 32 warps of 2 rows (64 registers) when one 206 KB CTA
// (head_dim 512) holds the SM, so that either way enough independent
// multiply-add chains are in flight.

template <int RPW>
__global__ void __launch_bounds__(32 * AP_R / RPW, RPW == 8 ? 2 : 1) attn_prefill_tiled(const AttnPrefillArgs a, int rowlen, int QB) {
  pdl_entry();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int d = a.d, dp = d + 4, G = a.Hq / a.Hkv, R = QB * G;
  int32_t* Qs = reinterpret_cast<int32_t*>(smem_raw);   // [AP_R][dp]
  int32_t* Ks = Qs + AP_R * dp;                          // [AP_TK][dp] (V tiles use [AP_TK][AP_CH+4])
  int32_t* Ws = Ks + AP_TK * dp;                         // [AP_R][AP_TK]
  __shared__ int32_t rmax[AP_R], ridx[AP_R];
  // query blocks in descending order: under a causal mask the last blocks
  // read the most keys, and starting them first keeps the final wave short
  const int kvh = blockIdx.x, i0 = (gridDim.y - 1 - blockIdx.y) * QB;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  auto row_query = [&](int r) { return i0 + (r % QB); };
  auto row_head = [&](int r) { return kvh * G + r / QB; };
  auto win_start = [&](int i) { return (a.window > 0 && i + 1 > a.window) ? i + 1 - a.window : 0; };
  const int klo = win_start(i0);
  const int khi = min(a.S, i0 + QB);
  // Q rows -> smem
  for (int e = threadIdx.x; e < AP_R * (d / 4); e += blockDim.x) {
    int r = e / (d / 4), c = e % (d / 4);
    int4 v = make_int4(0, 0, 0, 0);
    if (r < R && row_query(r) < a.S)
      v = reinterpret_cast<const int4*>(a.q + ((size_t)row_query(r) * a.Hq + row_head(r)) * d)[c];
    reinterpret_cast<int4*>(Qs + r * dp)[c] = v;
  }
  // ---- phase A: scores + first max
  int32_t bm[RPW], bi[RPW];
#pragma unroll
  for (int t = 0; t < RPW; ++t) { bm[t] = INT32_MIN; bi[t] = INT32_MAX; }
  const int rbase = warp * RPW;
  for (int kt = klo; kt < khi; kt += AP_TK) {
    __syncthreads();
    for (int e = threadIdx.x; e < AP_TK * (d / 4); e += blockDim.x) {
      int jj = e / (d / 4), c = e % (d / 4), j = kt + jj;
      int4 v = make_int4(0, 0, 0, 0);
      if (j < khi) v = reinterpret_cast<const int4*>(a.k_cache + ((size_t)kvh * a.cap + j) * d)[c];
      reinterpret_cast<int4*>(Ks + jj * dp)[c] = v;
    }
    __syncthreads();
    int64_t acc[RPW];
#pragma unroll
    for (int t = 0; t < RPW; ++t) acc[t] = 0;
    const int4* kr = reinterpret_cast<const int4*>(Ks + lane * dp);
    for (int c = 0; c < d / 4; ++c) {
      int4 kv = kr[c];
#pragma unroll
      for (int t = 0; t < RPW; ++t) {
        int4 qv = reinterpret_cast<const int4*>(Qs + (rbase + t) * dp)[c];
        acc[t] = dot4_acc(acc[t], kv, qv);
      }
    }
    const int j = kt + lane;
#pragma unroll
    for (int t = 0; t < RPW; ++t) {
      int r = rbase + t;
      if (r >= R) continue;
      int i = row_query(r);
      if (i >= a.S) continue;
      int st = win_start(i);
      if (j < st || j > i) continue;
      int32_t sc = requantize(acc[t]);
      a.scores[((size_t)row_head(r) * a.S + i) * rowlen + (j - st)] = sc;
      if (sc > bm[t] || bi[t] == INT32_MAX) { bm[t] = sc; bi[t] = j; }
    }
  }
#pragma unroll
  for (int t = 0; t < RPW; ++t) {
    int32_t v = bm[t], ix = bi[t];
    for (int o = 16; o > 0; o >>= 1) {
      int32_t v2 = __shfl_xor_sync(0xffffffffu, v, o), i2 = __shfl_xor_sync(0xffffffffu, ix, o);
      if (v2 > v || (v2 == v && i2 < ix)) { v = v2; ix = i2; }
    }
    if (lane == 0) { rmax[rbase + t] = v; ridx[rbase + t] = ix; }
  }
  __syncthreads();
  // ---- phase B: exact softmax weights per row (written over the scores)
  for (int t = 0; t < RPW; ++t) {
    int r = rbase + t;
    if (r >= R) break;
    int i = row_query(r);
    if (i >= a.S) continue;
    int st = win_start(i), n = i + 1 - st;
    int32_t* sc = a.scores + ((size_t)row_head(r) * a.S + i) * rowlen;
    int32_t mx = rmax[r];
    // four score loads in flight per lane (the scores sit in L2: one load
    // at a time left this phase waiting on L2 latency)
    constexpr int BU = 4;
    uint64_t sum = 0;
    for (int j0 = lane; j0 < n; j0 += 32 * BU) {
      int32_t v[BU];
#pragma unroll
      for (int u = 0; u < BU; ++u) v[u] = j0 + 32 * u < n ? sc[j0 + 32 * u] : 0;
#pragma unroll
      for (int u = 0; u < BU; ++u)
        if (j0 + 32 * u < n) sum += (uint64_t)exp_term(v[u], mx);
    }
    sum = (uint64_t)warp_sum64((int64_t)sum);
    int64_t wsum = 0;
    for (int j0 = lane; j0 < n; j0 += 32 * BU) {
      int32_t v[BU];
#pragma unroll
      for (int u = 0; u < BU; ++u) v[u] = j0 + 32 * u < n ? sc[j0 + 32 * u] : 0;
#pragma unroll
      for (int u = 0; u < BU; ++u)
        if (j0 + 32 * u < n) {
          const int32_t w = softmax_weight(exp_term(v[u], mx), (int64_t)sum);
          sc[j0 + 32 * u] = w;
          wsum += w;
        }
    }
    wsum = warp_sum64(wsum);
    __syncwarp();
    if (lane == 0) {
      int32_t res = sub_sat(kOneAct, wsum > INT32_MAX ? INT32_MAX : (int32_t)wsum);
      int m = ridx[r] - st;
      sc[m] = add_sat(sc[m], res);
    }
  }
  __syncthreads();
  // ---- phase C: out = requantize(sum_j w_j v_j), 128 output dims at a time
  const int rg = warp, dg = lane;
  const int cw = d < AP_CH ? d : AP_CH, cwp = cw + 4;
  // Double-buffered form: the Q tile region is free after phase A, so V and
  // weight tiles t + 1 load (cp.async, zero-filled outside the key range and
  // window) while tile t is multiplied.  Used when two buffers fit the
  // block's shared memory (every head_dim >= 64).
  const int vbuf = AP_TK * cwp + AP_R * AP_TK;  // ints per buffer: V tile, then weights
  const bool dbl = 2 * vbuf <= AP_R * dp + AP_TK * dp + AP_R * AP_TK;
  const int nkt = (khi - klo + AP_TK - 1) / AP_TK;
  for (int c0 = 0; dbl && c0 < d; c0 += AP_CH) {
    int64_t acc[RPW][4];
#pragma unroll
    for (int t = 0; t < RPW; ++t)
#pragma unroll
      for (int u = 0; u < 4; ++u) acc[t][u] = 0;
    auto issue = [&](int t) {
      int32_t* Vb = Qs + (t & 1) * vbuf;
      int32_t* Wb = Vb + AP_TK * cwp;
      const int kt = klo + t * AP_TK;
      for (int e = threadIdx.x; e < AP_TK * (cw / 4); e += blockDim.x) {
        const int jj = e / (cw / 4), c = e % (cw / 4), j = kt + jj;
        const int32_t* src = a.v_cache + ((size_t)kvh * a.cap + (j < khi ? j : klo)) * d + c0 + 4 * c;
        const unsigned sa = (unsigned)__cvta_generic_to_shared(Vb + jj * cwp + 4 * c);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sa), "l"(src), "r"(j < khi ? 16 : 0)
                     : "memory");
      }
      for (int e = threadIdx.x; e < AP_R * AP_TK; e += blockDim.x) {
        const int r = e / AP_TK, jj = e % AP_TK, j = kt + jj;
        const int32_t* src = a.scores;
        int bytes = 0;
        if (r < R) {
          const int i = row_query(r);
          if (i < a.S) {
            const int st = win_start(i);
            if (j >= st && j <= i) {
              src = a.scores + ((size_t)row_head(r) * a.S + i) * rowlen + (j - st);
              bytes = 4;
            }
          }
        }
        const unsigned sa = (unsigned)__cvta_generic_to_shared(Wb + r * AP_TK + jj);
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(sa), "l"(src), "r"(bytes) : "memory");
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    };
    __syncthreads();  // the region's previous users (phase A, the last chunk) are done
    if (nkt > 0) issue(0);
    for (int t = 0; t < nkt; ++t) {
      if (t + 1 < nkt) {
        issue(t + 1);
        asm volatile("cp.async.wait_group 1;" ::: "memory");
      } else {
        asm volatile("cp.async.wait_group 0;" ::: "memory");
      }
      __syncthreads();
      const int32_t* Vb = Qs + (t & 1) * vbuf;
      const int32_t* Wb = Vb + AP_TK * cwp;
      if (dg * 4 < cw) {
        for (int jj = 0; jj < AP_TK; ++jj) {
          const int4 v = reinterpret_cast<const int4*>(Vb + jj * cwp)[dg];
#pragma unroll
          for (int q = 0; q < RPW; ++q) {
            const int32_t w = Wb[(rg * RPW + q) * AP_TK + jj];
            acc[q][0] = mac_wide(acc[q][0], w, v.x);
            acc[q][1] = mac_wide(acc[q][1], w, v.y);
            acc[q][2] = mac_wide(acc[q][2], w, v.z);
            acc[q][3] = mac_wide(acc[q][3], w, v.w);
          }
        }
      }
      __syncthreads();  // buffer t & 1 is refilled by issue(t + 2)
    }
    if (dg * 4 < cw) {
#pragma unroll
      for (int q = 0; q < RPW; ++q) {
        const int r = rg * RPW + q;
        if (r >= R) continue;
        const int i = row_query(r);
        if (i >= a.S) continue;
        int32_t* o = a.out + ((size_t)i * a.Hq + row_head(r)) * d + c0 + dg * 4;
        o[0] = requantize(acc[q][0]);
        o[1] = requantize(acc[q][1]);
        o[2] = requantize(acc[q][2]);
        o[3] = requantize(acc[q][3]);
      }
    }
  }
  for (int c0 = 0; !dbl && c0 < d; c0 += AP_CH) {
    int64_t acc[RPW][4];
#pragma unroll
    for (int t = 0; t < RPW; ++t)
#pragma unroll
      for (int u = 0; u < 4; ++u) acc[t][u] = 0;
    for (int kt = klo; kt < khi; kt += AP_TK) {
      __syncthreads();
      for (int e = threadIdx.x; e < AP_TK * (cw / 4); e += blockDim.x) {
        int jj = e / (cw / 4), c = e % (cw / 4), j = kt + jj;
        int4 v = make_int4(0, 0, 0, 0);
        if (j < khi) v = reinterpret_cast<const int4*>(a.v_cache + ((size_t)kvh * a.cap + j) * d + c0)[c];
        reinterpret_cast<int4*>(Ks + jj * cwp)[c] = v;
      }
      for (int e = threadIdx.x; e < AP_R * AP_TK; e += blockDim.x) {
        int r = e / AP_TK, jj = e % AP_TK, j = kt + jj;
        int32_t w = 0;
        if (r < R) {
          int i = row_query(r);
          if (i < a.S) {
            int st = win_start(i);
            if (j >= st && j <= i) w = a.scores[((size_t)row_head(r) * a.S + i) * rowlen + (j - st)];
          }
        }
        Ws[r * AP_TK + jj] = w;
      }
      __syncthreads();
      if (dg * 4 < cw) {
        for (int jj = 0; jj < AP_TK; ++jj) {
          int4 v = reinterpret_cast<const int4*>(Ks + jj * cwp)[dg];
#pragma unroll
          for (int t = 0; t < RPW; ++t) {
            const int32_t w = Ws[(rg * RPW + t) * AP_TK + jj];
            acc[t][0] = mac_wide(acc[t][0], w, v.x);
            acc[t][1] = mac_wide(acc[t][1], w, v.y);
            acc[t][2] = mac_wide(acc[t][2], w, v.z);
            acc[t][3] = mac_wide(acc[t][3], w, v.w);
          }
        }
      }
    }
    if (dg * 4 < cw) {
#pragma unroll
      for (int t = 0; t < RPW; ++t) {
        int r = rg * RPW + t;
        if (r >= R) continue;
        int i = row_query(r);
        if (i >= a.S) continue;
        int32_t* o = a.out + ((size_t)i * a.Hq + row_head(r)) * d + c0 + dg * 4;
        o[0] = requantize(acc[t][0]);
        o[1] = requantize(acc[t][1]);
        o[2] = requantize(acc[t][2]);
        o[3] = requantize(acc[t][3]);
      }
    }
  }
}

void launch_attn_prefill(const AttnPrefillArgs& a, cudaStream_t s) {
  int rowlen = a.window > 0 ? (a.window < a.S ? a.window : a.S) : a.S;
  const int G = a.Hq / a.Hkv;
  size_t smem = ((size_t)AP_R * (a.d + 4) + (size_t)AP_TK * (a.d + 4) + (size_t)AP_R * AP_TK) * 4;
  if (a.d % 4 == 0 && a.d <= 512 && G <= AP_R && (a.d <= AP_CH || a.d % AP_CH == 0) && smem <= 220 * 1024) {
    int QB = AP_R / G;
    static bool configured = false;
    if (!configured) {
      cudaFuncSetAttribute(attn_prefill_tiled<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
      cudaFuncSetAttribute(attn_prefill_tiled<8>, cudaFuncAttributePreferredSharedMemoryCarveout,
                           cudaSharedmemCarveoutMaxShared);
      cudaFuncSetAttribute(attn_prefill_tiled<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
      cudaFuncSetAttribute(attn_prefill_tiled<2>, cudaFuncAttributePreferredSharedMemoryCarveout,
                           cudaSharedmemCarveoutMaxShared);
      configured = true;
    }
    dim3 grid(a.Hkv, (a.S + QB - 1) / QB);
    if (2 * (smem + 1024) <= 228 * 1024)  // two CTAs fit an SM's shared memory
      launch_k(attn_prefill_tiled<8>, dim3(grid), dim3(32 * AP_R / 8), smem, s, a, rowlen, QB);
    else
      launch_k(attn_prefill_tiled<2>, dim3(grid), dim3(32 * AP_R / 2), smem, s, a, rowlen, QB);
    return;
  }
  dim3 grid(a.Hq, a.S);
  launch_k(attn_prefill_kernel, dim3(grid), dim3(256), (size_t)a.d * 4, s, a, rowlen);
}

// ---------------------------------------------------------------------------
// embedding gather (io.rs:2446-2518), PLE inputs (prefill_prepare_aux)
// ---------------------------------------------------------------------------
__global__ void embed_kernel(const uint32_t* ids, DevMat emb, int32_t scale, int32_t* out, int32_t* err) {
  pdl_entry();
  const int s = blockIdx.x, H = emb.cols;
  uint32_t id = ids[s];
  if (id >= (uint32_t)emb.rows) {
    if (threadIdx.x == 0) atomicExch(err, 1);
    return;
  }
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    size_t off = (size_t)id * H + i;
    int32_t v = emb.width == 16 ? (int32_t) static_cast<const int16_t*>(emb.p)[off] : static_cast<const int32_t*>(emb.p)[off];
    out[(size_t)s * H + i] = mul_sat(v, scale);
  }
}
void launch_embed(const uint32_t* ids, int32_t S, const DevMat& emb, int32_t scale, int32_t* out, int32_t* err,
                  cudaStream_t s) {
  launch_k(embed_kernel, dim3(S), dim3(256), 0, s, ids, emb, scale, out, err);
}

__global__ void ple_kernel(const PleArgs a) {
  pdl_entry();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int32_t* vs = reinterpret_cast<int32_t*>(smem_raw);
  __shared__ uint64_t red[33];
  const int s = blockIdx.x, l = blockIdx.y, P = a.P;
  uint32_t id = a.ids[s];
  if (id >= (uint32_t)a.table.rows) {
    if (threadIdx.x == 0) atomicExch(a.err, 1);
    return;
  }
  const int32_t* pr = a.proj + (size_t)s * a.L * P + (size_t)l * P;
  for (int i = threadIdx.x; i < P; i += blockDim.x) vs[i] = mul_sat(pr[i], a.proj_scale);
  __syncthreads();
  int32_t sc = block_norm_scale(vs, P, a.eps, red);
  int32_t* o = a.out + ((size_t)l * a.S + s) * P;
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    int32_t nv = mul_sat(mul_sat(vs[i], sc), a.norm[i]);
    size_t off = (size_t)id * a.table.cols + (size_t)l * P + i;
    int32_t tv = a.table.width == 16 ? (int32_t) static_cast<const int16_t*>(a.table.p)[off]
                                     : static_cast<const int32_t*>(a.table.p)[off];
    o[i] = mul_sat(add_sat(mul_sat(tv, a.emb_scale), nv), a.in_scale);
  }
}
void launch_ple(const PleArgs& a, cudaStream_t s) {
  dim3 grid(a.S, a.L);
  launch_k(ple_kernel, dim3(grid), dim3(128), (size_t)a.P * 4, s, a);
}

// ---------------------------------------------------------------------------
// argmax_first (ops.rs:463): larger value wins; ties keep the lower index
// ---------------------------------------------------------------------------
__device__ __forceinline__ void better(int32_t& v, int32_t& i, int32_t v2, int32_t i2) {
  if (v2 > v || (v2 == v && i2 < i)) { v = v2; i = i2; }
}
__global__ void argmax_part_kernel(const int32_t* x, int n, int32_t* part) {
  pdl_entry();
  __shared__ int32_t sv[32], si[32];
  int32_t bv = INT32_MIN, bi = INT32_MAX;
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < n; j += gridDim.x * blockDim.x) better(bv, bi, x[j], j);
  for (int o = 16; o > 0; o >>= 1) {
    int32_t v2 = __shfl_xor_sync(0xffffffffu, bv, o), i2 = __shfl_xor_sync(0xffffffffu, bi, o);
    better(bv, bi, v2, i2);
  }
  if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) better(bv, bi, sv[w], si[w]);
    part[2 * blockIdx.x] = bv;
    part[2 * blockIdx.x + 1] = bi;
  }
}
__global__ void argmax_final_kernel(const int32_t* part, int blocks, uint32_t* idx) {
  pdl_entry();
  int32_t bv = INT32_MIN, bi = INT32_MAX;
  for (int b = 0; b < blocks; ++b) better(bv, bi, part[2 * b], part[2 * b + 1]);
  *idx = (uint32_t)bi;
}
void launch_argmax(const int32_t* x, int32_t n, int32_t* part, int32_t blocks, uint32_t* idx, cudaStream_t s) {
  launch_k(argmax_part_kernel, dim3(blocks), dim3(256), 0, s, x, n, part);
  launch_k(argmax_final_kernel, dim3(1), dim3(1), 0, s, part, blocks, idx);
}

// argmax_first of many rows at once.  Block (x, r) scans chunk x of row r
// (row r at rows[r] when rows is given, else at base + r * ld) and writes its
// first maximum as (value, idx0 + column) to part[(r * chunks + x) * 2].
__global__ void argmax_rows_part_kernel(const int32_t* const* rows, const int32_t* base, int32_t n, size_t ld,
                                        int32_t idx0, int32_t* part) {
  pdl_entry();
  __shared__ int32_t sv[32], si[32];
  const int r = blockIdx.y, chunks = gridDim.x;
  const int32_t* x = rows ? rows[r] : base + (size_t)r * ld;
  const int j0 = (int)((int64_t)n * blockIdx.x / chunks), j1 = (int)((int64_t)n * (blockIdx.x + 1) / chunks);
  int32_t bv = INT32_MIN, bi = INT32_MAX;
  for (int j = j0 + threadIdx.x; j < j1; j += blockDim.x) better(bv, bi, x[j], idx0 + j);
  for (int o = 16; o > 0; o >>= 1) {
    int32_t v2 = __shfl_xor_sync(0xffffffffu, bv, o), i2 = __shfl_xor_sync(0xffffffffu, bi, o);
    better(bv, bi, v2, i2);
  }
  if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) better(bv, bi, sv[w], si[w]);
    part[((size_t)r * chunks + blockIdx.x) * 2] = bv;
    part[((size_t)r * chunks + blockIdx.x) * 2 + 1] = bi;
  }
}
// Row r's token from the pairs of `world` row blocks laid out
// [world][B][chunks][2] (the vocab-sharded ranks' pairs after an all-gather;
// world 1 for one GPU).  Comparing (value, index) keeps argmax_first's
// lowest-index tie-break whatever the order of the pairs.
__global__ void argmax_rows_final_kernel(const int32_t* part, int32_t world, int32_t B, int32_t chunks,
                                         uint32_t* tokens) {
  pdl_entry();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= B) return;
  int32_t bv = INT32_MIN, bi = INT32_MAX;
  for (int w = 0; w < world; ++w)
    for (int x = 0; x < chunks; ++x) {
      const int32_t* p = part + (((size_t)w * B + r) * chunks + x) * 2;
      better(bv, bi, p[0], p[1]);
    }
  tokens[r] = (uint32_t)bi;
}
void launch_argmax_rows(const int32_t* const* rows, const int32_t* base, int32_t B, int32_t n, size_t ld,
                        int32_t idx0, int32_t chunks, int32_t* part, cudaStream_t s) {
  launch_k(argmax_rows_part_kernel, dim3(chunks, B), dim3(256), 0, s, rows, base, n, ld, idx0, part);
}
void launch_argmax_rows_final(const int32_t* part, int32_t world, int32_t B, int32_t chunks, uint32_t* tokens,
                              cudaStream_t s) {
  launch_k(argmax_rows_final_kernel, dim3((B + 127) / 128), dim3(128), 0, s, part, world, B, chunks, tokens);
}
__global__ void softcap_kernel(int32_t* x, int n, int32_t cap) {
  pdl_entry();
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < n; j += gridDim.x * blockDim.x) x[j] = softcap_act(x[j], cap);
}
void launch_softcap(int32_t* x, int32_t n, int32_t cap, cudaStream_t s) {
  launch_k(softcap_kernel, dim3((n + 255) / 256 < 1024 ? (n + 255) / 256 : 1024), dim3(256), 0, s, x, n, cap);
}

// ---------------------------------------------------------------------------
// misc
// ---------------------------------------------------------------------------
__global__ void add_i32_rows_kernel(int32_t* const* p, int32_t n, int32_t v) {
  pdl_entry();
  for (int i = threadIdx.x; i < n; i += blockDim.x) *p[i] += v;
}
void launch_add_i32_rows(int32_t* const* p, int32_t n, int32_t v, cudaStream_t s) {
  launch_k(add_i32_rows_kernel, dim3(1), dim3(256), 0, s, p, n, v);
}
// Row r of src -> dst[r] + off; with cap > 0 each value passes through
// softcap_act on the way (the logit softcap fused into the copy).
__global__ void scatter_rows_kernel(const int32_t* src, int32_t n, int32_t* const* dst, size_t off, int32_t cap) {
  pdl_entry();
  const int r = blockIdx.y;
  const int32_t* sr = src + (size_t)r * n;
  int32_t* dr = dst[r] + off;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int32_t v = sr[i];
    dr[i] = cap > 0 ? softcap_act(v, cap) : v;
  }
}
void launch_scatter_rows(const int32_t* src, int32_t rows, int32_t n, int32_t* const* dst, size_t off,
                         cudaStream_t s, int32_t cap) {
  // about 8 values per thread, every row spread over several blocks
  const int bx = std::max(1, std::min(1024, (n + 2047) / 2048));
  launch_k(scatter_rows_kernel, dim3(bx, rows), dim3(256), 0, s, src, n, dst, off, cap);
}

__global__ void requantize_rows_kernel(const int64_t* x, size_t n, int32_t* y) {
  pdl_entry();
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    y[i] = requantize(x[i]);
}
__global__ void tp_signal_kernel(const TpPeerFlags peers, int world, int rank, uint32_t value) {
  pdl_entry();
  const int r = threadIdx.x;
  if (r < world && r != rank && peers.f[r]) {
    // the sums the preceding kernels wrote are visible system-wide before the flag
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(peers.f[r] + rank), "r"(value) : "memory");
  }
}
void launch_tp_signal(const TpPeerFlags& peers, int32_t world, int32_t rank, uint32_t value, cudaStream_t s) {
  launch_k(tp_signal_kernel, dim3(1), dim3(32), 0, s, peers, (int)world, (int)rank, value);
}
void launch_requantize_rows(const int64_t* x, size_t n, int32_t* y, cudaStream_t s) {
  const int blocks = (int)std::min<size_t>((n + 255) / 256, (size_t)sm_count() * 4);
  launch_k(requantize_rows_kernel, dim3(blocks > 0 ? blocks : 1), dim3(256), 0, s, x, n, y);
}
__global__ void gather_vocab_kernel(const int32_t* src, int32_t world, int32_t rows, int32_t vl, int32_t* const* dst) {
  pdl_entry();
  const int r = blockIdx.y;
  int32_t* d = dst[r];
  const size_t n = (size_t)world * vl;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t w = i / vl, j = i % vl;
    d[i] = src[(w * rows + r) * vl + j];
  }
}
void launch_gather_vocab(const int32_t* src, int32_t world, int32_t rows, int32_t vl, int32_t* const* dst,
                         cudaStream_t s) {
  launch_k(gather_vocab_kernel, dim3(64, rows), dim3(256), 0, s, src, world, rows, vl, dst);
}

__global__ void add_i32_kernel(int32_t* p, int32_t v) {
  pdl_entry(); *p += v; }
void launch_add_i32(int32_t* p, int32_t v, cudaStream_t s) { launch_k(add_i32_kernel, dim3(1), dim3(1), 0, s, p, v); }
void launch_copy_rows(const int32_t* src, int32_t* dst, size_t n, cudaStream_t s) {
  cudaMemcpyAsync(dst, src, n * 4, cudaMemcpyDeviceToDevice, s);
}

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
__global__ void synth_kernel(void* dst, int width, int rank, int64_t n, int64_t cols, uint64_t key) {
  pdl_entry();
  const uint64_t GOLD = 0x9E3779B97F4A7C15ull;
  int64_t bound = cols > 0 ? (int64_t)(0x7fffffffLL / cols) : 0;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    uint64_t z = mix64(key + (uint64_t)(i + 1) * GOLD);
    int32_t v;
    if (rank == 1) v = 32768 + (int32_t)(z >> 48);
    else if (width == 16) v = (int32_t)(z >> 48) - 32768;
    else v = (int32_t)((int64_t)(z % (uint64_t)(2 * bound + 1)) - bound);
    if (width == 16) static_cast<int16_t*>(dst)[i] = (int16_t)v;
    else static_cast<int32_t*>(dst)[i] = v;
  }
}
void launch_synth(void* dst, int32_t width, int32_t rank, int64_t n, int64_t cols, uint64_t key, cudaStream_t s) {
  int64_t blocks = (n + 255) / 256;
  if (blocks > 65536) blocks = 65536;
  if (blocks < 1) blocks = 1;
  launch_k(synth_kernel, dim3((unsigned)blocks), dim3(256), 0, s, dst, width, rank, n, cols, key);
}

}  // namespace rdet
