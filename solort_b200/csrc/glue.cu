// Layer glue of the decode / verify / prefill step around the attention: the residual add fused
// with the next RMSNorm, and SiLU(gate) * up. Reference: src/solort/model/cuda_graph_executor.py
// _rmsnorm :25-28 (fp32 math: x * rsqrt(mean(x^2) + eps), times the weight, cast back) on the input
// and post-attention norms and the final norm, the residual adds of the layer loop, and the MLP's
// F.silu(gate) * up. In the reference these are ~18 small torch kernels per layer; here three.
//
// add_rmsnorm_kernel: one CTA per row. x_out = bf16(x + delta) (delta optional), then
// h = bf16((x_out * rsqrt(mean(x_out^2) + eps)) * w) with the mean over fp32 values (a warp-shuffle
// and shared-memory tree, so its last bit can differ from torch's reduction order).
// silu_mul_kernel: out = bf16(bf16(g / (1 + exp(-g))) * u), the rounding of F.silu then a bf16 mul.
#include <math.h>

#include "common.cuh"
#include "host_util.h"

namespace solort {
namespace glue {

constexpr int kNormThreads = 256;

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
  uint4 u;
  u.x = pack_bf16x2(v[0], v[1]);
  u.y = pack_bf16x2(v[2], v[3]);
  u.z = pack_bf16x2(v[4], v[5]);
  u.w = pack_bf16x2(v[6], v[7]);
  return u;
}

struct NormParams {
  const bf16* x;
  const bf16* delta;  // optional
  const bf16* w;
  bf16* x_out;        // written when delta != nullptr
  bf16* h_out;
  int64_t x_st, d_st, xo_st, h_st;
  int hidden;
  float eps;
};

// Chunks of 8 values per thread; up to kMaxChunks per thread stay in registers between the two
// passes (hidden <= 256 * 8 * kMaxChunks = 16384).
constexpr int kMaxChunks = 8;

__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(const NormParams p) {
  __shared__ float red[kNormThreads / 32];
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int row = blockIdx.x, tid = threadIdx.x;
  const int chunks = p.hidden / 8;
  float v[kMaxChunks][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kMaxChunks; ++k) {
    const int c = tid + k * kNormThreads;
    if (c < chunks) {
      unpack8(*reinterpret_cast<const uint4*>(p.x + row * p.x_st + c * 8), v[k]);
      if (p.delta) {
        float d[8];
        unpack8(*reinterpret_cast<const uint4*>(p.delta + row * p.d_st + c * 8), d);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[k][i] = bf(v[k][i] + d[i]);
        *reinterpret_cast<uint4*>(p.x_out + row * p.xo_st + c * 8) = pack8(v[k]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += v[k][i] * v[k][i];
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot += red[i];
  const float r = rsqrtf(tot * (1.f / static_cast<float>(p.hidden)) + p.eps);  // mean as sum * (1/N)
#pragma unroll
  for (int k = 0; k < kMaxChunks; ++k) {
    const int c = tid + k * kNormThreads;
    if (c < chunks) {
      float w[8], y[8];
      unpack8(*reinterpret_cast<const uint4*>(p.w + c * 8), w);
#pragma unroll
      for (int i = 0; i < 8; ++i) y[i] = (v[k][i] * r) * w[i];
      *reinterpret_cast<uint4*>(p.h_out + row * p.h_st + c * 8) = pack8(y);
    }
  }
}

struct SiluParams {
  const bf16* gu;  // [rows, 2 * inter]: gate then up
  bf16* out;       // [rows, inter]
  int64_t gu_st, o_st;
  int inter;
};

__global__ void __launch_bounds__(256) silu_mul_kernel(const SiluParams p) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int row = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;  // chunk of 8
  if (c * 8 >= p.inter) return;
  float g[8], u[8], y[8];
  unpack8(*reinterpret_cast<const uint4*>(p.gu + row * p.gu_st + c * 8), g);
  unpack8(*reinterpret_cast<const uint4*>(p.gu + row * p.gu_st + p.inter + c * 8), u);
#pragma unroll
  for (int i = 0; i < 8; ++i) y[i] = bf(g[i] / (1.f + expf(-g[i]))) * u[i];
  *reinterpret_cast<uint4*>(p.out + row * p.o_st + c * 8) = pack8(y);
}

inline cudaLaunchConfig_t pdl_cfg(dim3 grid, dim3 block, cudaStream_t s, cudaLaunchAttribute* at) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = s;
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cfg;
}

}  // namespace glue
}  // namespace solort

using namespace solort;

extern "C" int solort_attn_add_rmsnorm(const SolortAddRmsNormArgs* a, void* stream) {
  if (!a || !a->x || !a->weight || !a->h_out || (a->delta && !a->x_out))
    return SOLORT_ERR_INVALID_ARGUMENT;
  if (a->rows <= 0 || a->hidden <= 0 || (a->hidden & 7) ||
      a->hidden > glue::kNormThreads * 8 * glue::kMaxChunks)
    return SOLORT_ERR_UNSUPPORTED;
  const int64_t st = a->x_stride | a->delta_stride | a->x_out_stride | a->h_out_stride;
  if ((st & 7) || !aligned(a->x, 16) || !aligned(a->h_out, 16) || !aligned(a->weight, 16) ||
      (a->delta && (!aligned(a->delta, 16) || !aligned(a->x_out, 16))))
    return SOLORT_ERR_INVALID_ARGUMENT;
  DeviceInfo di;
  int rc = current_device_info(&di);
  if (rc != SOLORT_OK) return rc;
  glue::NormParams p{};
  p.x = static_cast<const bf16*>(a->x);
  p.delta = static_cast<const bf16*>(a->delta);
  p.w = static_cast<const bf16*>(a->weight);
  p.x_out = static_cast<bf16*>(a->x_out);
  p.h_out = static_cast<bf16*>(a->h_out);
  p.x_st = a->x_stride;
  p.d_st = a->delta_stride;
  p.xo_st = a->x_out_stride;
  p.h_st = a->h_out_stride;
  p.hidden = a->hidden;
  p.eps = a->eps;
  cudaLaunchAttribute at[1];
  cudaLaunchConfig_t cfg = glue::pdl_cfg(dim3(a->rows), dim3(glue::kNormThreads),
                                         static_cast<cudaStream_t>(stream), at);
  if (cudaLaunchKernelEx(&cfg, glue::add_rmsnorm_kernel, p) != cudaSuccess) return SOLORT_ERR_CUDA;
  return launch_status();
}

extern "C" int solort_attn_silu_mul(const SolortSiluMulArgs* a, void* stream) {
  if (!a || !a->gate_up || !a->out) return SOLORT_ERR_INVALID_ARGUMENT;
  if (a->rows <= 0 || a->rows > 65535 || a->inter <= 0 || (a->inter & 7))
    return SOLORT_ERR_UNSUPPORTED;
  if (((a->gate_up_stride | a->out_stride) & 7) || !aligned(a->gate_up, 16) || !aligned(a->out, 16))
    return SOLORT_ERR_INVALID_ARGUMENT;
  DeviceInfo di;
  int rc = current_device_info(&di);
  if (rc != SOLORT_OK) return rc;
  glue::SiluParams p{};
  p.gu = static_cast<const bf16*>(a->gate_up);
  p.out = static_cast<bf16*>(a->out);
  p.gu_st = a->gate_up_stride;
  p.o_st = a->out_stride;
  p.inter = a->inter;
  const int chunks = a->inter / 8;
  cudaLaunchAttribute at[1];
  cudaLaunchConfig_t cfg = glue::pdl_cfg(dim3((chunks + 255) / 256, a->rows), dim3(256),
                                         static_cast<cudaStream_t>(stream), at);
  if (cudaLaunchKernelEx(&cfg, glue::silu_mul_kernel, p) != cudaSuccess) return SOLORT_ERR_CUDA;
  return launch_status();
}
