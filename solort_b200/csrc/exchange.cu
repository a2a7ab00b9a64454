// Receive side of the sequence-sharded decode exchange, and the exchange buffers.
//
// Every rank's merge kernel (decode.cu, exchange mode) stores its partial rows (O fp32 [rows][128],
// then LSE [rows]) straight into a slot of every rank's receive buffer over NVLink and raises one
// flag per row there with a system-scope release. exchange_merge_kernel, on each rank, gives one
// warp to each output row: lanes 0..R-1 each wait (acquire, bounded by one second) for the row's
// flag from one rank, the warp then reads the R partial rows from its own memory, combines them
// by log-sum-exp and writes the bf16 row, and finally clears the R flags for the next use of the
// slots. No collective library runs on this path and no kernel loads from peer memory: peers only
// store into it.
//
// The buffers are plain cudaMalloc allocations exported with CUDA IPC handles, so each process
// maps its peers' buffers with cudaIpcOpenMemHandle: point-to-point mappings only.
#include <math.h>
#include <string.h>

#include "common.cuh"
#include "host_util.h"

namespace solort {

__device__ unsigned g_exchange_status;

namespace xch {

constexpr int kHD = 128;
constexpr int kRowsPerCta = 4;  // one warp per output row
constexpr unsigned kDevErrPeerTimeout = 1u << 3;

struct Params {
  const float* slots;  // rank s: slots + s * slot_stride
  unsigned* flags;     // rank s: flags + s * flag_stride
  int64_t slot_stride, flag_stride;
  int num_ranks;
  int rows;
  int q_len, nh;
  bf16* out;
  int64_t o_sb, o_st, o_sh;
};

__global__ void __launch_bounds__(kRowsPerCta * 32) exchange_merge_kernel(const Params p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kRowsPerCta + warp;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (row >= p.rows) return;

  // Wait for this row's partial from every rank.
  bool ok = true;
  if (lane < p.num_ranks) {
    const unsigned* f = p.flags + lane * p.flag_stride + row;
    const unsigned long long t0 = globaltimer_ns();
    unsigned v = 0;
    for (unsigned i = 0;; ++i) {
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
      if (v != 0u) break;
      if ((i & 63u) == 0u && globaltimer_ns() - t0 > kWaitLimitNs) {
        ok = false;
        break;
      }
    }
  }
  if (!__all_sync(0xffffffffu, ok)) {
    if (lane == 0) atomicOr(&g_exchange_status, kDevErrPeerTimeout);
    return;  // flags stay as they are: the host sees the status bit
  }
  __syncwarp();

  // Log-sum-exp combine of the R partial rows (R <= 8): lane l holds dims 4l..4l+3.
  float lse[SOLORT_MAX_RANKS];
  float4 o[SOLORT_MAX_RANKS];
  float M = -INFINITY;
#pragma unroll
  for (int s = 0; s < SOLORT_MAX_RANKS; ++s) {
    if (s < p.num_ranks) {
      const float* slot = p.slots + s * p.slot_stride;
      lse[s] = __ldcg(slot + static_cast<int64_t>(p.rows) * kHD + row);
      o[s] = __ldcg(reinterpret_cast<const float4*>(slot + static_cast<int64_t>(row) * kHD) + lane);
      M = fmaxf(M, lse[s]);
    }
  }
  float D = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int s = 0; s < SOLORT_MAX_RANKS; ++s) {
    if (s < p.num_ranks && lse[s] != -INFINITY) {
      const float w = __expf(lse[s] - M);
      D += w;
      acc.x += w * o[s].x;
      acc.y += w * o[s].y;
      acc.z += w * o[s].z;
      acc.w += w * o[s].w;
    }
  }
  const float inv = D > 0.f ? __frcp_rn(D) : 0.f;
  const int h = row % p.nh, t = (row / p.nh) % p.q_len, b = row / (p.nh * p.q_len);
  bf16* dst = p.out + b * p.o_sb + t * p.o_st + h * p.o_sh + lane * 4;
  uint2 pk;
  pk.x = pack_bf16x2(acc.x * inv, acc.y * inv);
  pk.y = pack_bf16x2(acc.z * inv, acc.w * inv);
  *reinterpret_cast<uint2*>(dst) = pk;

  // Every lane's reads are done: clear the flags for the next use of these slots.
  __syncwarp();
  if (lane < p.num_ranks) p.flags[lane * p.flag_stride + row] = 0u;
}

}  // namespace xch

int read_exchange_status(unsigned* flags) {
  unsigned v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_exchange_status, sizeof(v)) != cudaSuccess)
    return SOLORT_ERR_CUDA;
  if (v && cudaMemcpyToSymbol(g_exchange_status, &zero, sizeof(zero)) != cudaSuccess)
    return SOLORT_ERR_CUDA;
  *flags |= v;
  return SOLORT_OK;
}

}  // namespace solort

using namespace solort;

extern "C" int solort_attn_exchange_merge(const SolortExchangeMergeArgs* a, void* stream) {
  if (!a || !a->slots || !a->flags || !a->out) return SOLORT_ERR_INVALID_ARGUMENT;
  if (a->head_dim != xch::kHD) return SOLORT_ERR_UNSUPPORTED;
  if (a->num_ranks < 1 || a->num_ranks > SOLORT_MAX_RANKS) return SOLORT_ERR_INVALID_ARGUMENT;
  if (a->batch <= 0 || a->q_len <= 0 || a->num_qo_heads <= 0) return SOLORT_ERR_INVALID_ARGUMENT;
  if (!aligned(a->slots, 16) || !aligned(a->flags, 4) || !aligned(a->out, 8) ||
      (a->out_stride_batch | a->out_stride_token | a->out_stride_head) & 3)
    return SOLORT_ERR_INVALID_ARGUMENT;
  const int64_t rows = static_cast<int64_t>(a->batch) * a->q_len * a->num_qo_heads;
  if (rows > (1ll << 30)) return SOLORT_ERR_UNSUPPORTED;
  if (a->slot_stride < rows * (xch::kHD + 1) || (a->slot_stride & 3) || a->flag_stride < rows)
    return SOLORT_ERR_INVALID_ARGUMENT;
  DeviceInfo di;
  int rc = current_device_info(&di);
  if (rc != SOLORT_OK) return rc;
  xch::Params p{};
  p.slots = a->slots;
  p.flags = a->flags;
  p.slot_stride = a->slot_stride;
  p.flag_stride = a->flag_stride;
  p.num_ranks = a->num_ranks;
  p.rows = static_cast<int>(rows);
  p.q_len = a->q_len;
  p.nh = a->num_qo_heads;
  p.out = static_cast<bf16*>(a->out);
  p.o_sb = a->out_stride_batch;
  p.o_st = a->out_stride_token;
  p.o_sh = a->out_stride_head;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((rows + xch::kRowsPerCta - 1) / xch::kRowsPerCta));
  cfg.blockDim = dim3(xch::kRowsPerCta * 32);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, xch::exchange_merge_kernel, p) != cudaSuccess)
    return SOLORT_ERR_CUDA;
  return launch_status();
}

extern "C" int solort_attn_exchange_buffer_create(size_t bytes, void** ptr, void* ipc_handle) {
  if (!ptr || !ipc_handle || bytes == 0) return SOLORT_ERR_INVALID_ARGUMENT;
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  DeviceInfo di;
  int rc = current_device_info(&di);
  if (rc != SOLORT_OK) return rc;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return SOLORT_ERR_CUDA;
  if (cudaMemset(p, 0, bytes) != cudaSuccess) {
    cudaFree(p);
    return SOLORT_ERR_CUDA;
  }
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return SOLORT_ERR_IPC;
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return SOLORT_OK;
}

extern "C" int solort_attn_exchange_buffer_open(const void* ipc_handle, void** ptr) {
  if (!ptr || !ipc_handle) return SOLORT_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return SOLORT_ERR_IPC;
  *ptr = p;
  return SOLORT_OK;
}

extern "C" int solort_attn_exchange_buffer_close(void* ptr) {
  if (!ptr) return SOLORT_ERR_INVALID_ARGUMENT;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? SOLORT_OK : SOLORT_ERR_IPC;
}

extern "C" int solort_attn_exchange_buffer_destroy(void* ptr) {
  if (!ptr) return SOLORT_ERR_INVALID_ARGUMENT;
  return cudaFree(ptr) == cudaSuccess ? SOLORT_OK : SOLORT_ERR_CUDA;
}
