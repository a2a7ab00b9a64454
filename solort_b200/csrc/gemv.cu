// Weight-streaming projection for the decode step: y[t, n] = sum_k act[t, k] W[n, k] for a handful
// of token rows (t <= 8) against a bf16 weight W [N, K] (a torch Linear weight). At t <= 8 a
// projection is a pure weight stream (every weight byte is used t times), so it is built for HBM
// bandwidth, not tensor cores. The activation is staged once per CTA in shared memory, as
//   mode 0: a itself;
//   mode 1: bf16(bf16(silu(g)) * u) of a fused gate|up row (the reference MLP's F.silu(gate) * up,
//           src/solort/model/cuda_graph_executor.py), so the down projection needs no extra launch;
//   mode 2: RMSNorm(x + delta) * weight (the reference's _rmsnorm, :25-28, after the residual add),
//           so each residual add + norm of the layer loop runs inside the next projection. The sum
//           of squares is accumulated in exactly the order of the add_rmsnorm kernel, so the two
//           paths give the same bits; CTA 0 also writes bf16(x + delta) to x_out.
//
// Layout: eight warps per CTA, one output row per warp (or per pair of warps, below) at a time; a
// grid of four CTAs per SM (64 registers; fewer fit when t * K * 2 bytes of staged activations
// are large, and the grid then runs in waves) strides over groups of rows, so the staging is
// amortised over a CTA's groups. Each lane keeps eight 16-byte weight loads in flight, and the next
// group's first batch is issued before the current row is reduced. The first batch is issued
// before the kernel waits for its predecessor on the stream (programmatic dependent launch); W
// must therefore not be written by the kernel just before this one (model weights are not).
//
// Measured alternatives not kept (whole decode step): a persistent CTA per SM streaming its rows
// with bulk async copies into a ~200 KB shared-memory ring (10-15% slower: the large-smem CTA
// cannot overlap the kernels before and after it), a double-buffered register pipeline (half the
// resident warps), ten loads per lane in flight, the whole MLP as one launch with a grid
// barrier between gate_up and down (the barrier cost more than the kernel boundary), and an
// even split of each CTA's rows over its warps as equal runs of 16-byte chunks (warps ending
// mid-row, partials added in shared memory) to remove the warps left with an extra row: slower
// on every projection alone (gate_up 19.3 -> 26.5 us, down 18.2 -> 21.1 us) and 371 -> 310
// tokens/s; the row-per-warp streams keep more loads in flight than the balance gains.
#include <atomic>
#include <math.h>

#include <algorithm>

#include "common.cuh"
#include "host_util.h"

namespace solort {
namespace gemv {

constexpr int kWarps = 8;      // = output rows per group
constexpr int kThreads = kWarps * 32;
constexpr int kUnroll = 8;     // 16-byte weight loads in flight per lane
constexpr int kMaxT = 8;
constexpr int kCtasPerSm = 4;
constexpr int kMaxStageBytes = 160 * 1024;

struct Params {
  const bf16* a;         // mode 0: [t, K]; mode 1: [t, 2K] gate|up; mode 2: residual x [t, K]
  int64_t a_st;
  const bf16* w;         // [N, K]
  int64_t w_st;
  bf16* y;               // [t, N]
  int64_t y_st;
  int t, n, k;
  int mode;
  const bf16* delta;     // mode 2 (optional): added to x before the norm
  int64_t delta_st;
  const bf16* norm_w;    // mode 2: [K]
  bf16* x_out;           // mode 2 with delta: bf16(x + delta)
  int64_t x_out_st;
  float eps;
};

__device__ __forceinline__ float bf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ void unpack8(const uint4& u, float (&v)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __low2float(h[i]);
    v[2 * i + 1] = __high2float(h[i]);
  }
}

__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  return make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                    pack_bf16x2(v[6], v[7]));
}

__device__ __forceinline__ void dot8(float& acc, const uint4& w, const uint4& a) {
  const __nv_bfloat162* wh = reinterpret_cast<const __nv_bfloat162*>(&w);
  const __nv_bfloat162* ah = reinterpret_cast<const __nv_bfloat162*>(&a);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 wf = __bfloat1622float2(wh[i]);
    const float2 af = __bfloat1622float2(ah[i]);
    acc = fmaf(wf.x, af.x, acc);
    acc = fmaf(wf.y, af.y, acc);
  }
}

// Stage act [T][K] in shared memory. Rows past t repeat row 0 (their results are never stored).
template <int T>
__device__ __forceinline__ void stage_activations(const Params& p, bf16* act, float* red) {
  const int chunks = p.k / 8, tid = threadIdx.x;
  if (p.mode != 2) {
    for (int idx = tid; idx < T * chunks; idx += kThreads) {
      const int tt = idx / chunks, c = idx - tt * chunks;
      const int src = tt < p.t ? tt : 0;
      uint4 v;
      if (p.mode == 0) {
        v = __ldcg(reinterpret_cast<const uint4*>(p.a + src * p.a_st + c * 8));
      } else {
        float g[8], u[8], o[8];
        unpack8(__ldcg(reinterpret_cast<const uint4*>(p.a + src * p.a_st + c * 8)), g);
        unpack8(__ldcg(reinterpret_cast<const uint4*>(p.a + src * p.a_st + p.k + c * 8)), u);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = bf(g[i] / (1.f + expf(-g[i]))) * u[i];
        v = pack8(o);
      }
      *reinterpret_cast<uint4*>(act + tt * p.k + c * 8) = v;
    }
    __syncthreads();
    return;
  }
  // mode 2: per row, x (+ delta) rounded to bf16, its fp32 sum of squares (per thread over
  // chunks tid, tid + 256, ..., then a shuffle tree, then the warps in order: the add_rmsnorm
  // kernel's order), r = rsqrt(mean + eps), act = bf16((v * r) * w).
  const bool write_x = p.x_out != nullptr && blockIdx.x == 0;
#pragma unroll 1
  for (int tt = 0; tt < T; ++tt) {
    const int src = tt < p.t ? tt : 0;
    float ss = 0.f;
    for (int c = tid; c < chunks; c += kThreads) {
      float v[8];
      unpack8(__ldcg(reinterpret_cast<const uint4*>(p.a + src * p.a_st + c * 8)), v);
      if (p.delta) {
        float d[8];
        unpack8(__ldcg(reinterpret_cast<const uint4*>(p.delta + src * p.delta_st + c * 8)), d);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = bf(v[i] + d[i]);
      }
      const uint4 packed = pack8(v);
      *reinterpret_cast<uint4*>(act + tt * p.k + c * 8) = packed;
      if (write_x && tt < p.t) *reinterpret_cast<uint4*>(p.x_out + tt * p.x_out_st + c * 8) = packed;
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kWarps; ++i) tot += red[i];
    const float r = rsqrtf(tot * (1.f / static_cast<float>(p.k)) + p.eps);
    for (int c = tid; c < chunks; c += kThreads) {
      float v[8], w[8];
      unpack8(*reinterpret_cast<const uint4*>(act + tt * p.k + c * 8), v);
      unpack8(*reinterpret_cast<const uint4*>(p.norm_w + c * 8), w);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = (v[i] * r) * w[i];
      *reinterpret_cast<uint4*>(act + tt * p.k + c * 8) = pack8(v);
    }
    __syncthreads();  // act complete; red free for the next row
  }
}

// S warps share each output row (S = 1 or 2, a template parameter so the S = 1 kernel carries no
// split bookkeeping; four warps per row measured slower over the whole decode step): warp w takes
// row w / S of its group, chunk range part w % S of it.
template <int S>
struct RowSplit {
  int part, c_begin, c_end;
  __device__ __forceinline__ RowSplit(int warp, int chunks) {
    part = S > 1 ? warp % S : 0;
    const int spp = S > 1 ? ((chunks + 31) / 32 + S - 1) / S : 0;  // whole 32-chunk slots
    c_begin = S > 1 ? part * spp * 32 : 0;
    c_end = S > 1 ? min(chunks, c_begin + spp * 32) : chunks;
  }
};

// The first batch of loads of this warp's part of `row` (zeros past the matrix).
template <int S>
__device__ __forceinline__ void load_first(const Params& p, const RowSplit<S>& rs, int row,
                                           uint4 (&wv)[kUnroll]) {
  const int lane = threadIdx.x & 31;
  const bf16* wrow = p.w + static_cast<int64_t>(row) * p.w_st;
#pragma unroll
  for (int u = 0; u < kUnroll; ++u) {
    const int c = rs.c_begin + lane + u * 32;
    wv[u] = (row < p.n && c < rs.c_end) ? *reinterpret_cast<const uint4*>(wrow + c * 8)
                                        : make_uint4(0u, 0u, 0u, 0u);
  }
}

// Rows of groups blockIdx.x, + gridDim.x, ... against the staged activations; `wv` holds the first
// group's first batch on entry.
template <int T, int S>
__device__ __forceinline__ void stream_rows(const Params& p, const bf16* act,
                                            uint4 (&wv)[kUnroll]) {
  __shared__ float part_sum[S > 1 ? 2 : 1][kWarps][T];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const RowSplit<S> rs(warp, p.k / 8);
  constexpr int kRows = kWarps / S;  // rows per group
  const int groups = (p.n + kRows - 1) / kRows;
  constexpr int kStep = 32 * kUnroll;
  int buf = 0;
  for (int g = blockIdx.x; g < groups; g += gridDim.x) {
    const int row = g * kRows + warp / S;
    const bf16* wrow = p.w + static_cast<int64_t>(row) * p.w_st;
    float acc[T];
#pragma unroll
    for (int tt = 0; tt < T; ++tt) acc[tt] = 0.f;
    if (row < p.n) {
      for (int c0 = rs.c_begin; c0 < rs.c_end; c0 += kStep) {
        if (c0 > rs.c_begin) {
#pragma unroll
          for (int u = 0; u < kUnroll; ++u) {
            const int c = c0 + lane + u * 32;
            wv[u] = c < rs.c_end ? *reinterpret_cast<const uint4*>(wrow + c * 8)
                                 : make_uint4(0u, 0u, 0u, 0u);
          }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int c = c0 + lane + u * 32;
          if (c < rs.c_end) {
#pragma unroll
            for (int tt = 0; tt < T; ++tt)
              dot8(acc[tt], wv[u], *reinterpret_cast<const uint4*>(act + tt * p.k + c * 8));
          }
        }
      }
    }
    // The next group's first batch goes out before this row is reduced and stored.
    load_first<S>(p, rs, (g + gridDim.x) * kRows + warp / S, wv);
    if (S == 1) {
      if (row < p.n) {
#pragma unroll
        for (int tt = 0; tt < T; ++tt) {
          float v = acc[tt];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
          if (lane == 0 && tt < p.t) p.y[tt * p.y_st + row] = __float2bfloat16_rn(v);
        }
      }
    } else {
      // The row's partials meet in shared memory (double-buffered by group, one barrier per
      // group) and its first warp sums them in warp order.
      float mine = 0.f;
#pragma unroll
      for (int tt = 0; tt < T; ++tt) {
        float v = acc[tt];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == tt) mine = v;
      }
      if (lane < T) part_sum[buf][warp][lane] = mine;
      asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory");
      if (rs.part == 0 && row < p.n && lane < p.t) {
        float v = 0.f;
#pragma unroll
        for (int j = 0; j < S; ++j) v += part_sum[buf][warp + j][lane];
        p.y[lane * p.y_st + row] = __float2bfloat16_rn(v);
      }
      buf ^= 1;
    }
  }
}

template <int T, int S>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) gemv_kernel(const Params p) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float red[kWarps];
  bf16* act = reinterpret_cast<bf16*>(smem);  // [T][K]
  const int warp = threadIdx.x >> 5;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  uint4 wv[kUnroll];
  load_first<S>(p, RowSplit<S>(warp, p.k / 8), blockIdx.x * (kWarps / S) + warp / S, wv);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  stage_activations<T>(p, act, red);
  stream_rows<T, S>(p, act, wv);
}

template <int T, int S>
int launch(const Params& p, size_t smem, int grid, cudaStream_t stream) {
  static std::atomic<unsigned> configured{0};  // one bit per device ordinal < 32
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return SOLORT_ERR_CUDA;
  if (dev >= 32 || !(configured.load(std::memory_order_acquire) & (1u << dev))) {
    if (cudaFuncSetAttribute(gemv_kernel<T, S>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kMaxStageBytes) != cudaSuccess)
      return SOLORT_ERR_CUDA;
    if (dev < 32) configured.fetch_or(1u << dev, std::memory_order_release);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, gemv_kernel<T, S>, p) != cudaSuccess) return SOLORT_ERR_CUDA;
  return launch_status();
}

// Two warps share a row when it spans more than one batch of loads and there are too few rows to
// keep every warp of a resident wave busy twice over (qkv, o_proj, down of Qwen3-4B; a row of
// 9728 is five serial batches for one warp while half the resident warps idle). Whole decode step
// of the Qwen3-4B shape: 359 -> 371 tokens/s.
inline int default_split(int n, int k, int sm_count) {
  const int spr = (k / 8 + 31) / 32;
  return (spr > kUnroll && n < 2 * kWarps * sm_count * kCtasPerSm) ? 2 : 1;
}

template <int T>
int launch_split(const Params& p, size_t smem, int split, int grid_cap, cudaStream_t s) {
  const int rows = kWarps / split;
  const int grid = std::min((p.n + rows - 1) / rows, grid_cap);
  return split == 2 ? launch<T, 2>(p, smem, grid, s) : launch<T, 1>(p, smem, grid, s);
}

inline bool overlaps(const void* a, int64_t a_bytes, const void* b, int64_t b_bytes) {
  const uintptr_t x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
  return x < y + static_cast<uintptr_t>(b_bytes) && y < x + static_cast<uintptr_t>(a_bytes);
}

}  // namespace gemv

}  // namespace solort

using namespace solort;

extern "C" int solort_attn_gemv(const SolortGemvArgs* a, void* stream_v) {
  if (!a || !a->a || !a->w || !a->y) return SOLORT_ERR_INVALID_ARGUMENT;
  if (a->t <= 0 || a->t > gemv::kMaxT || a->n <= 0 || a->k <= 0 || (a->k & 7) || a->mode < 0 ||
      a->mode > 2)
    return SOLORT_ERR_UNSUPPORTED;
  const int T = a->t <= 1 ? 1 : a->t <= 2 ? 2 : a->t <= 4 ? 4 : 8;
  const size_t smem = static_cast<size_t>(T) * a->k * 2;
  if (smem > static_cast<size_t>(gemv::kMaxStageBytes)) return SOLORT_ERR_UNSUPPORTED;
  if (((a->a_stride | a->w_stride) & 7) || !aligned(a->a, 16) || !aligned(a->w, 16) ||
      !aligned(a->y, 2) || a->w_stride < a->k ||
      a->a_stride < (a->mode == 1 ? 2 : 1) * static_cast<int64_t>(a->k) || a->y_stride < a->n)
    return SOLORT_ERR_INVALID_ARGUMENT;
  if (a->mode == 2) {
    if (!a->norm_weight || !aligned(a->norm_weight, 16) || (a->delta && !a->x_out) ||
        (a->x_out && !a->delta))
      return SOLORT_ERR_INVALID_ARGUMENT;
    if (a->delta) {
      if (((a->delta_stride | a->x_out_stride) & 7) || !aligned(a->delta, 16) ||
          !aligned(a->x_out, 16) || a->delta_stride < a->k || a->x_out_stride < a->k)
        return SOLORT_ERR_INVALID_ARGUMENT;
      // x_out is written by one CTA while the others still read x and delta.
      const int64_t span = static_cast<int64_t>(a->t - 1);
      const int64_t xo_bytes = (span * a->x_out_stride + a->k) * 2;
      if (gemv::overlaps(a->x_out, xo_bytes, a->a, (span * a->a_stride + a->k) * 2) ||
          gemv::overlaps(a->x_out, xo_bytes, a->delta, (span * a->delta_stride + a->k) * 2))
        return SOLORT_ERR_INVALID_ARGUMENT;
    }
  }
  DeviceInfo di;
  int rc = current_device_info(&di);
  if (rc != SOLORT_OK) return rc;
  gemv::Params p{};
  p.a = static_cast<const bf16*>(a->a);
  p.a_st = a->a_stride;
  p.w = static_cast<const bf16*>(a->w);
  p.w_st = a->w_stride;
  p.y = static_cast<bf16*>(a->y);
  p.y_st = a->y_stride;
  p.t = a->t;
  p.n = a->n;
  p.k = a->k;
  p.mode = a->mode;
  if (a->mode == 2) {
    p.delta = static_cast<const bf16*>(a->delta);
    p.delta_st = a->delta_stride;
    p.norm_w = static_cast<const bf16*>(a->norm_weight);
    p.x_out = static_cast<bf16*>(a->x_out);
    p.x_out_st = a->x_out_stride;
    p.eps = a->eps;
  }
  const int split = gemv::default_split(a->n, a->k, di.sm_count);
  const int cap = di.sm_count * gemv::kCtasPerSm;
  cudaStream_t s = static_cast<cudaStream_t>(stream_v);
  switch (T) {
    case 1: return gemv::launch_split<1>(p, smem, split, cap, s);
    case 2: return gemv::launch_split<2>(p, smem, split, cap, s);
    case 4: return gemv::launch_split<4>(p, smem, split, cap, s);
    default: return gemv::launch_split<8>(p, smem, split, cap, s);
  }
}
