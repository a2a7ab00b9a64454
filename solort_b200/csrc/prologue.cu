// Attention prologue: per-head QK-RMSNorm + rotate-half RoPE of the fused QKV projection, the
// normalised queries written for the attention kernels, and this step's K / V rows appended to
// the cache (static rows at their positions, or paged slots through a block table).
//
// Reference (src/solort/model/cuda_graph_executor.py): _rmsnorm :25-28 (fp32 math, cast back, then
// times the weight), _cos_sin :95-98 (bf16 tables), _rope :100-102 (x*cos + rotate_half(x)*sin in
// bf16), the per-layer sequence :176-179 (decode), :120-123 (prefill) and :257-260 (verify), and
// the paged slot mapping of src/solort/cache/kv_cache.py:136-149 (slot = bt[p // P] * P + p % P).
//
// One warp per (token, head) row of 128 values; lane l holds dims 4l..4l+3. The rotate-half partner
// of dim d is d +- 64, i.e. lane l ^ 16. Rounding follows the reference step by step: the norm's
// product is rounded to bf16, then x*cos and rotate_half(x)*sin are each rounded to bf16 before their
// bf16 sum. The fp32 sum of squares is a warp-shuffle tree, so its last bit can differ from torch's
// reduction order. V rows are copied unchanged. One launch replaces the reference's ~28 small ops
// (norm pieces, RoPE pieces, index_copy_) of a layer.
#include <math.h>

#include "common.cuh"
#include "host_util.h"

namespace solort {
namespace pro {

constexpr unsigned kDevErrSlotRange = 1u << 4;  // solort_attn_kv_store skipped a slot past the arena
__device__ unsigned g_store_status;

constexpr int kHD = 128;
constexpr int kWarpsPerCta = 8;

struct Params {
  const bf16* qkv;
  int64_t qkv_st;
  int t, nh, nkv;
  const bf16* qn;
  const bf16* kn;
  float eps;
  const bf16* cos;
  const bf16* sin;
  int64_t rope_st;
  int rope_rows;
  const int64_t* pos;
  bf16* q_out;
  int64_t qo_st, qo_sh;
  bf16* k_cache;
  bf16* v_cache;
  int64_t kv_st, kv_sh, kv_sp;
  int kv_capacity;  // static: rows in the cache; paged: num_pages * page_size
  const int32_t* block_table;
  int page_size, page_shift;
};

__device__ __forceinline__ float bf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ void load4(const bf16* p, float (&v)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&u.x);
  const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
  v[0] = __low2float(a);
  v[1] = __high2float(a);
  v[2] = __low2float(b);
  v[3] = __high2float(b);
}

__device__ __forceinline__ void store4(bf16* p, const float (&v)[4]) {
  uint2 u;
  u.x = pack_bf16x2(v[0], v[1]);
  u.y = pack_bf16x2(v[2], v[3]);
  *reinterpret_cast<uint2*>(p) = u;
}

// Destination of cache row (token position `position`, kv head h), or nullptr past the cache.
__device__ __forceinline__ int64_t cache_offset(const Params& p, long long position, int h) {
  if (position < 0 || position >= p.kv_capacity) return -1;
  if (!p.block_table) return position * p.kv_st + h * p.kv_sh;
  const int page = p.block_table[position >> p.page_shift];
  const int row = static_cast<int>(position & (p.page_size - 1));
  return static_cast<int64_t>(page) * p.kv_sp + row * p.kv_st + h * p.kv_sh;
}

__global__ void __launch_bounds__(kWarpsPerCta * 32) prologue_kernel(const Params p) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int lane = threadIdx.x & 31;
  const int heads = p.nh + 2 * p.nkv;
  const int w = blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
  if (w >= p.t * heads) return;
  const int tok = w / heads, head = w % heads;
  const long long position = p.pos[0] + tok;
  const bf16* src = p.qkv + tok * p.qkv_st + head * kHD + lane * 4;
  float x[4];
  load4(src, x);

  if (head >= p.nh + p.nkv) {  // V: appended unchanged
    const int h = head - p.nh - p.nkv;
    const int64_t off = cache_offset(p, position, h);
    if (off >= 0) store4(p.v_cache + off + lane * 4, x);
    return;
  }

  // RMSNorm in fp32 (warp-shuffle sum of squares), times the weight, rounded to bf16.
  float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = rsqrtf(ss * (1.f / kHD) + p.eps);
  const bool is_q = head < p.nh;
  float wgt[4];
  load4((is_q ? p.qn : p.kn) + lane * 4, wgt);
  float y[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) y[i] = bf((x[i] * r) * wgt[i]);

  // Rotate-half RoPE with the bf16 tables: bf16(bf16(y*cos) + bf16(rot(y)*sin)).
  float c[4], s[4];
  const int64_t rr = position < p.rope_rows ? position : p.rope_rows - 1;
  load4(p.cos + rr * p.rope_st + lane * 4, c);
  load4(p.sin + rr * p.rope_st + lane * 4, s);
  float out[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float partner = __shfl_xor_sync(0xffffffffu, y[i], 16);
    const float rot = lane < 16 ? -partner : partner;
    out[i] = bf(bf(y[i] * c[i]) + bf(rot * s[i]));
  }

  if (is_q) {
    store4(p.q_out + tok * p.qo_st + head * p.qo_sh + lane * 4, out);
  } else {
    const int64_t off = cache_offset(p, position, head - p.nh);
    if (off >= 0) store4(p.k_cache + off + lane * 4, out);
  }
}

}  // namespace pro
}  // namespace solort

using namespace solort;

extern "C" int solort_attn_qk_norm_rope_append(const SolortPrologueArgs* a, void* stream) {
  if (!a || !a->qkv || !a->q_norm_weight || !a->k_norm_weight || !a->cos || !a->sin || !a->pos ||
      !a->q_out || !a->k_cache || !a->v_cache)
    return SOLORT_ERR_INVALID_ARGUMENT;
  if (a->head_dim != pro::kHD) return SOLORT_ERR_UNSUPPORTED;
  if (a->num_tokens <= 0 || a->num_qo_heads <= 0 || a->num_kv_heads <= 0 || a->rope_rows <= 0 ||
      a->kv_capacity <= 0)
    return SOLORT_ERR_INVALID_ARGUMENT;
  // 8-byte vector accesses everywhere: pointers 8-aligned, strides multiples of 4 elements.
  const int64_t strides = a->qkv_stride_token | a->rope_stride | a->q_out_stride_token |
                          a->q_out_stride_head | a->kv_stride_token | a->kv_stride_head |
                          a->kv_stride_page;
  if ((strides & 3) || !aligned(a->qkv, 8) || !aligned(a->q_out, 8) || !aligned(a->k_cache, 8) ||
      !aligned(a->v_cache, 8) || !aligned(a->cos, 8) || !aligned(a->sin, 8) ||
      !aligned(a->q_norm_weight, 8) || !aligned(a->k_norm_weight, 8))
    return SOLORT_ERR_INVALID_ARGUMENT;
  int shift = 0;
  if (a->block_table) {
    const int P = a->page_size;
    if (P < 1 || (P & (P - 1)) != 0) return SOLORT_ERR_INVALID_ARGUMENT;
    while ((1 << shift) < P) ++shift;
  }
  DeviceInfo di;
  int rc = current_device_info(&di);
  if (rc != SOLORT_OK) return rc;
  pro::Params p{};
  p.qkv = static_cast<const bf16*>(a->qkv);
  p.qkv_st = a->qkv_stride_token;
  p.t = a->num_tokens;
  p.nh = a->num_qo_heads;
  p.nkv = a->num_kv_heads;
  p.qn = static_cast<const bf16*>(a->q_norm_weight);
  p.kn = static_cast<const bf16*>(a->k_norm_weight);
  p.eps = a->eps;
  p.cos = static_cast<const bf16*>(a->cos);
  p.sin = static_cast<const bf16*>(a->sin);
  p.rope_st = a->rope_stride;
  p.rope_rows = a->rope_rows;
  p.pos = a->pos;
  p.q_out = static_cast<bf16*>(a->q_out);
  p.qo_st = a->q_out_stride_token;
  p.qo_sh = a->q_out_stride_head;
  p.k_cache = static_cast<bf16*>(a->k_cache);
  p.v_cache = static_cast<bf16*>(a->v_cache);
  p.kv_st = a->kv_stride_token;
  p.kv_sh = a->kv_stride_head;
  p.kv_sp = a->kv_stride_page;
  p.kv_capacity = a->kv_capacity;
  p.block_table = a->block_table;
  p.page_size = a->block_table ? a->page_size : 1;
  p.page_shift = shift;
  const int64_t warps = static_cast<int64_t>(a->num_tokens) *
                        (a->num_qo_heads + 2 * a->num_kv_heads);
  if (warps > (1ll << 30)) return SOLORT_ERR_UNSUPPORTED;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((warps + pro::kWarpsPerCta - 1) / pro::kWarpsPerCta));
  cfg.blockDim = dim3(pro::kWarpsPerCta * 32);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, pro::prologue_kernel, p) != cudaSuccess) return SOLORT_ERR_CUDA;
  return launch_status();
}

// ------------------------------------------------------------------------------------------------
// Slot-mapped KV store (the HF bridge's mirror into SoloRT's paged arena). The reference writes
// one token at a time from Python (src/solort/cache/kv_cache.py:230-235: k_cache[layer, page,
// offset].copy_(k_tokens[i]) for each slot); here one warp moves one (token, head) row of K and
// one of V, 256 bytes each as a 16-byte load and store per lane over 16 lanes.
// ------------------------------------------------------------------------------------------------
namespace solort {
namespace pro {

struct StoreParams {
  const bf16* key;
  const bf16* value;
  int64_t src_st, src_sh;
  int t, nkv;
  const int64_t* slots;
  bf16* k_pages;
  bf16* v_pages;
  int64_t dst_sp, dst_st, dst_sh;
  int page_shift, page_size;
  long long slot_limit;  // num_pages * page_size
};

__global__ void __launch_bounds__(kWarpsPerCta * 32) kv_store_kernel(const StoreParams p) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int lane = threadIdx.x & 31;
  const int w = blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
  if (w >= p.t * p.nkv) return;
  const int tok = w / p.nkv, h = w % p.nkv;
  const long long slot = p.slots[tok];
  if (slot < 0 || slot >= p.slot_limit) {
    if (lane == 0) atomicOr(&g_store_status, kDevErrSlotRange);
    return;
  }
  const long long page = slot >> p.page_shift;
  const int row = static_cast<int>(slot & (p.page_size - 1));
  const int64_t dst = page * p.dst_sp + row * p.dst_st + h * p.dst_sh;
  const int64_t src = tok * p.src_st + h * p.src_sh;
  // lanes 0-15 move the K row, lanes 16-31 the V row: 16 lanes x 16 bytes = 128 bf16 each
  const int part = lane & 15;
  const bf16* from = (lane < 16 ? p.key : p.value) + src + part * 8;
  bf16* to = (lane < 16 ? p.k_pages : p.v_pages) + dst + part * 8;
  *reinterpret_cast<uint4*>(to) = *reinterpret_cast<const uint4*>(from);
}

}  // namespace pro

int read_store_status(unsigned* flags) {
  unsigned v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, pro::g_store_status, sizeof(v)) != cudaSuccess)
    return SOLORT_ERR_CUDA;
  if (v && cudaMemcpyToSymbol(pro::g_store_status, &zero, sizeof(zero)) != cudaSuccess)
    return SOLORT_ERR_CUDA;
  *flags |= v;
  return SOLORT_OK;
}

}  // namespace solort

extern "C" int solort_attn_kv_store(const SolortKVStoreArgs* a, void* stream) {
  if (!a || !a->key || !a->value || !a->slots || !a->k_pages || !a->v_pages)
    return SOLORT_ERR_INVALID_ARGUMENT;
  if (a->head_dim != pro::kHD) return SOLORT_ERR_UNSUPPORTED;
  if (a->num_tokens < 0 || a->num_kv_heads <= 0 || a->num_pages <= 0)
    return SOLORT_ERR_INVALID_ARGUMENT;
  const int P = a->page_size;
  if (P < 1 || (P & (P - 1)) != 0) return SOLORT_ERR_INVALID_ARGUMENT;
  // 16-byte vector accesses: pointers 16-aligned, strides multiples of 8 elements.
  const int64_t strides = a->src_stride_token | a->src_stride_head | a->dst_stride_page |
                          a->dst_stride_token | a->dst_stride_head;
  if ((strides & 7) || !aligned(a->key, 16) || !aligned(a->value, 16) ||
      !aligned(a->k_pages, 16) || !aligned(a->v_pages, 16) || !aligned(a->slots, 8))
    return SOLORT_ERR_INVALID_ARGUMENT;
  if (a->num_tokens == 0) return SOLORT_OK;
  DeviceInfo di;
  int rc = current_device_info(&di);
  if (rc != SOLORT_OK) return rc;
  const int64_t warps = static_cast<int64_t>(a->num_tokens) * a->num_kv_heads;
  if (warps > (1ll << 30)) return SOLORT_ERR_UNSUPPORTED;
  pro::StoreParams p{};
  p.key = static_cast<const bf16*>(a->key);
  p.value = static_cast<const bf16*>(a->value);
  p.src_st = a->src_stride_token;
  p.src_sh = a->src_stride_head;
  p.t = a->num_tokens;
  p.nkv = a->num_kv_heads;
  p.slots = a->slots;
  p.k_pages = static_cast<bf16*>(a->k_pages);
  p.v_pages = static_cast<bf16*>(a->v_pages);
  p.dst_sp = a->dst_stride_page;
  p.dst_st = a->dst_stride_token;
  p.dst_sh = a->dst_stride_head;
  int shift = 0;
  while ((1 << shift) < P) ++shift;
  p.page_shift = shift;
  p.page_size = P;
  p.slot_limit = static_cast<long long>(a->num_pages) * P;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((warps + pro::kWarpsPerCta - 1) / pro::kWarpsPerCta));
  cfg.blockDim = dim3(pro::kWarpsPerCta * 32);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, pro::kv_store_kernel, p) != cudaSuccess) return SOLORT_ERR_CUDA;
  return launch_status();
}
