// Receive side of the sequence-sharded decode exchange, and the exchange buffers.
//
// Every rank's merge kernel (decode.cu, exchange mode) stores its partial rows (O [rows][128],
// then LSE [rows]) straight into a slot of every rank's receive buffer over NVLink, as 64-bit
// words whose high half is an arrival mark and whose low half is the float (one single-copy-atomic
// store per word, the scheme of NCCL's low-latency protocol). exchange_merge_kernel, on each rank,
// gives one warp to each output row: every lane polls its own words of the R slots (relaxed,
// system-scope loads of this GPU's memory, bounded by one second) until all carry the mark, the
// warp combines the R partials by log-sum-exp and writes the bf16 row, and the lanes then zero the
// words they read for the next use of the slots. No fence, flag or collective library is on this
// path, and no kernel loads from peer memory: peers only store into it.
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
  unsigned long long* slots;  // rank s: slots + s * slot_stride words
  int64_t slot_stride;
  int num_ranks;
  int rows;
  int q_len, nh;
  bf16* out;
  int64_t o_sb, o_st, o_sh;
};

__device__ __forceinline__ unsigned long long load_word(const unsigned long long* w) {
  unsigned long long x;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(x) : "l"(w) : "memory");
  return x;
}

__global__ void __launch_bounds__(kRowsPerCta * 32) exchange_merge_kernel(const Params p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kRowsPerCta + warp;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (row >= p.rows) return;

  // Lane l's words in slot s: O dims 4l..4l+3 of this row, and the row's LSE.
  float o[SOLORT_MAX_RANKS][4];
  float lse[SOLORT_MAX_RANKS];
  bool ok = true;
  const unsigned long long t0 = globaltimer_ns();
#pragma unroll
  for (int s = 0; s < SOLORT_MAX_RANKS; ++s) {
    if (s >= p.num_ranks) break;
    const unsigned long long* slot = p.slots + s * p.slot_stride;
    const unsigned long long* wo = slot + static_cast<int64_t>(row) * kHD + lane * 4;
    const unsigned long long* wl = slot + static_cast<int64_t>(p.rows) * kHD + row;
    for (unsigned i = 0;; ++i) {
      const unsigned long long x0 = load_word(wo), x1 = load_word(wo + 1), x2 = load_word(wo + 2),
                               x3 = load_word(wo + 3), xl = load_word(wl);
      if ((x0 >> 32) & (x1 >> 32) & (x2 >> 32) & (x3 >> 32) & (xl >> 32)) {
        o[s][0] = __uint_as_float(static_cast<unsigned>(x0));
        o[s][1] = __uint_as_float(static_cast<unsigned>(x1));
        o[s][2] = __uint_as_float(static_cast<unsigned>(x2));
        o[s][3] = __uint_as_float(static_cast<unsigned>(x3));
        lse[s] = __uint_as_float(static_cast<unsigned>(xl));
        break;
      }
      if ((i & 15u) == 0u && globaltimer_ns() - t0 > kWaitLimitNs) {
        ok = false;
        break;
      }
    }
    if (!ok) break;
  }
  if (!__all_sync(0xffffffffu, ok)) {
    if (lane == 0) atomicOr(&g_exchange_status, kDevErrPeerTimeout);
    return;  // the slots stay as they are: the host sees the status bit
  }

  // Log-sum-exp combine of the R partial rows: lane l holds dims 4l..4l+3.
  float M = -INFINITY;
#pragma unroll
  for (int s = 0; s < SOLORT_MAX_RANKS; ++s)
    if (s < p.num_ranks) M = fmaxf(M, lse[s]);
  float D = 0.f, a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
  for (int s = 0; s < SOLORT_MAX_RANKS; ++s) {
    if (s < p.num_ranks && lse[s] != -INFINITY) {
      const float w = __expf(lse[s] - M);
      D += w;
      a0 += w * o[s][0];
      a1 += w * o[s][1];
      a2 += w * o[s][2];
      a3 += w * o[s][3];
    }
  }
  const float inv = D > 0.f ? __frcp_rn(D) : 0.f;
  const int h = row % p.nh, t = (row / p.nh) % p.q_len, b = row / (p.nh * p.q_len);
  bf16* dst = p.out + b * p.o_sb + t * p.o_st + h * p.o_sh + lane * 4;
  uint2 pk;
  pk.x = pack_bf16x2(a0 * inv, a1 * inv);
  pk.y = pack_bf16x2(a2 * inv, a3 * inv);
  *reinterpret_cast<uint2*>(dst) = pk;

  // Zero the words this warp read (every lane has its values): the slots are ready for reuse.
  __syncwarp();
  for (int s = 0; s < p.num_ranks; ++s) {
    unsigned long long* slot = p.slots + s * p.slot_stride;
    unsigned long long* wo = slot + static_cast<int64_t>(row) * kHD + lane * 4;
    *reinterpret_cast<ulonglong2*>(wo) = make_ulonglong2(0ull, 0ull);
    *reinterpret_cast<ulonglong2*>(wo + 2) = make_ulonglong2(0ull, 0ull);
    if (lane == 0) slot[static_cast<int64_t>(p.rows) * kHD + row] = 0ull;
  }
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
  if (!a || !a->slots || !a->out) return SOLORT_ERR_INVALID_ARGUMENT;
  if (a->head_dim != xch::kHD) return SOLORT_ERR_UNSUPPORTED;
  if (a->num_ranks < 1 || a->num_ranks > SOLORT_MAX_RANKS) return SOLORT_ERR_INVALID_ARGUMENT;
  if (a->batch <= 0 || a->q_len <= 0 || a->num_qo_heads <= 0) return SOLORT_ERR_INVALID_ARGUMENT;
  if (!aligned(a->slots, 16) || !aligned(a->out, 8) ||
      (a->out_stride_batch | a->out_stride_token | a->out_stride_head) & 3)
    return SOLORT_ERR_INVALID_ARGUMENT;
  const int64_t rows = static_cast<int64_t>(a->batch) * a->q_len * a->num_qo_heads;
  if (rows > (1ll << 30)) return SOLORT_ERR_UNSUPPORTED;
  if (a->slot_stride < rows * (xch::kHD + 1) || (a->slot_stride & 1))
    return SOLORT_ERR_INVALID_ARGUMENT;
  DeviceInfo di;
  int rc = current_device_info(&di);
  if (rc != SOLORT_OK) return rc;
  xch::Params p{};
  p.slots = reinterpret_cast<unsigned long long*>(a->slots);
  p.slot_stride = a->slot_stride;
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
