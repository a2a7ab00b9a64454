// Causal GQA prefill on the 5th-generation tensor cores (tcgen05 + TMEM) for sm_100a.
//
// One CTA computes one 128-row tile of queries for one query head against the KV head of its
// group (GQA without expanding K/V: the query heads of a group read the same K/V tiles, which
// stay in L2). 384 threads with fixed roles:
//   warp 0, lane 0   TMA: the Q tile once, then K tiles into a 2-stage ring
//   warp 2, lane 0   TMA: V tiles into a 2-stage ring
//   warp 1           allocates 512 TMEM columns (S/P double buffer + O); lane 0 issues every
//                    tcgen05.mma: S_j = Q K_j^T into S[j&1] (A, B from shared memory), then
//                    O += P_{j-1} V_{j-1} with P read from TMEM (A operand in tensor memory)
//   warps 4..7, 8..11  two softmax warp groups; thread r of group g owns query row r and key
//                    columns [64g, 64g+64): it reads its S slice from TMEM (tcgen05.ld), the two
//                    groups exchange row maxima through shared memory, then it writes its slice
//                    of P as packed bf16 back over S (tcgen05.st), rescales its O columns when
//                    the row max grows by more than 2^8, and finally normalises and stores O.
// P aliases the S buffer it came from: the tensor core runs one CTA's MMAs in issue order, and
// QK_{j+2} (which overwrites that buffer) is issued only after PV_j (which reads P_j).
// Tiles above the causal diagonal are skipped; only diagonal / partial tiles are masked.
// Completion is tracked with mbarriers (TMA transaction bytes, tcgen05.commit, thread arrivals);
// every wait is bounded and a shared abort flag lets all roles leave together.
//
// Semantics: the reference's causal SDPA over the padded prompt (src/solort/model/
// cuda_graph_executor.py:124-130) and the HF bridge's bottom-right causal alignment when q_len <
// kv_len (src/solort/backends/transformers_flashinfer.py:182-193): query i sees keys
// j <= kv_len - q_len + i.
#include <atomic>
#include <math.h>

#include "common.cuh"
#include "host_util.h"

namespace solort {

__device__ unsigned g_prefill_status;

namespace pre {

constexpr int kHD = 128;
constexpr int kBM = 128;                     // query rows per CTA
constexpr int kBN = 128;                     // keys per tile
constexpr int kTileBytes = kBN * kHD * 2;    // 32 KB: one K or V tile (two 64-dim swizzled halves)
constexpr int kHalf = kTileBytes / 2;        // 16 KB
constexpr int kStages = 2;
constexpr int kThreads = 384;
constexpr int kSoftmaxThreads = 256;         // two warp groups
constexpr int kTmemCols = 512;
constexpr float kRescaleLog2 = 8.f;          // lazy rescale threshold (factor 256)
constexpr int kPingPongMinTiles = 16;        // 128-row query tiles from which two go per CTA
constexpr int kStageRow = kHD * 2 + 16;      // bytes per row of the output tile staged for the store

// shared memory map (offsets from a 1024-aligned base)
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kTileBytes;
constexpr int kOffV = kOffK + kStages * kTileBytes;
constexpr int kOffX = kOffV + kStages * kTileBytes;  // row-max exchange [2][2][128] + sums [2][128]
constexpr int kOffBar = kOffX + 3 * 2 * kBM * 4;
constexpr int kSmemBytes = 1024 + kOffBar + 256;

struct Params {
  bf16* out;
  int64_t o_st, o_sh;
  int q_len, kv_len, nh, group;
  int q_tiles;
  int causal;
  int q_tok_coord, kv_tok_coord;  // 1: map coords (d, tok, head); 2: (d, head, tok)
  float scale_log2;
};

// Barrier indices
enum {
  kBarQ = 0,
  kBarKFull = 1,                     // +stage
  kBarKEmpty = kBarKFull + kStages,
  kBarVFull = kBarKEmpty + kStages,
  kBarVEmpty = kBarVFull + kStages,
  kBarSFull = kBarVEmpty + kStages,  // +buffer (2): QK_j committed
  kBarPFull = kBarSFull + 2,         // 256 arrivals: P_j written to TMEM
  kBarPVDone = kBarPFull + 1,        // PV_j committed
  kBarXMax = kBarPVDone + 1,         // +parity*4 + warp pair (8), 64 arrivals: row-max exchange
  kBarXSum = kBarXMax + 8,           // 256 arrivals: final row-sum exchange
  kBarOStaged = kBarXSum + 1,        // 256 arrivals: the output tile staged in shared memory
  kNumBars = kBarOStaged + 1
};

__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;  // descriptor version for sm_100
  d |= static_cast<uint64_t>(2u) << 61;  // 128-byte swizzle
  return d;
}

// kind::f16 instruction descriptor: fp32 accumulate, bf16 A and B, M = 128, N = 128.
constexpr uint32_t kIdescQK = (1u << 4) | (1u << 7) | (1u << 10) | ((kBN >> 3) << 17) |
                              ((kBM >> 4) << 24);                // A, B K-major
constexpr uint32_t kIdescPV = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) |
                              ((kHD >> 3) << 17) | ((kBM >> 4) << 24);  // B (V) MN-major

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

// A operand read from tensor memory (K-major: row m in lane m, two 16-bit values per column).
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate));
}

// Packed fp32 pairs (sm_100): one instruction computes two lanes.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
  return d;
}
__device__ __forceinline__ void f2_unpack(uint64_t d, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(d));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void tmem_st32u(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31, %32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Bounded wait that also gives up as soon as another role has aborted.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(addr, parity)) return true;
    if ((i & 127u) == 0u) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        atomicOr(&g_prefill_status, kDevErrBarrierTimeout);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // issue / commit counts, read by the abort drain: [0] K tiles, [1] V tiles, [2] QK, [3] PV
  volatile int* counts = reinterpret_cast<volatile int*>(tmem_slot + 2);
  const uint32_t sbase = smem_u32(smem);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // heaviest (last) query tiles first
  const int q_tile = p.q_tiles - 1 - static_cast<int>(blockIdx.x) / p.nh;
  const int head = static_cast<int>(blockIdx.x) % p.nh;
  const int kvh = head / p.group;
  const int q0 = q_tile * kBM;
  const int offset = p.kv_len - p.q_len;  // bottom-right alignment
  const int kv_tiles_all = (p.kv_len + kBN - 1) / kBN;
  int n_tiles = kv_tiles_all;
  if (p.causal) {
    const int last_row = min(q0 + kBM, p.q_len) - 1;
    const int last_key = offset + last_row;  // >= 0 whenever q_len <= kv_len
    n_tiles = min(kv_tiles_all, last_key / kBN + 1);
  }

  if (tid == 0) {
    for (int i = 0; i < kNumBars; ++i) {
      const uint32_t count =
          (i == kBarPFull || i == kBarXSum || i == kBarOStaged) ? kSoftmaxThreads
          : (i >= kBarXMax && i < kBarXMax + 8) ? 64u
                                                 : 1u;
      mbar_init(&bars[i], count);
    }
    *abort_flag = 0;
    for (int i = 0; i < 4; ++i) counts[i] = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Launched as a programmatic dependent: everything above (barriers, TMEM) overlaps the previous
  // kernel's tail; Q, K, V and the output are touched only after it has finished. The next kernel
  // may launch only now, once every CTA holds its TMEM: a dependent CTA that took the columns
  // first would wait on this grid while this CTA waited on the columns.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS[2] = {tmem, tmem + kBN};
  const uint32_t tO = tmem + 2 * kBN;

  if (warp == 0 && lane == 0) {
    // ---- Q + K producer ----
    prefetch_tensormap(&tmQ);
    prefetch_tensormap(&tmK);
    mbar_arrive_expect_tx(&bars[kBarQ], kTileBytes);
    for (int h = 0; h < 2; ++h) {
      const int c1 = p.q_tok_coord == 1 ? q0 : head, c2 = p.q_tok_coord == 1 ? head : q0;
      tma_load_3d(smem + kOffQ + h * kHalf, &tmQ, &bars[kBarQ], h * 64, c1, c2);
    }
    for (int j = 0; j < n_tiles; ++j) {
      const int s = j % kStages;
      if (j >= kStages && !wait_bar(&bars[kBarKEmpty + s], ((j / kStages) - 1) & 1, abort_flag)) break;
      mbar_arrive_expect_tx(&bars[kBarKFull + s], kTileBytes);
      for (int h = 0; h < 2; ++h) {
        const int t = j * kBN;
        const int c1 = p.kv_tok_coord == 1 ? t : kvh, c2 = p.kv_tok_coord == 1 ? kvh : t;
        tma_load_3d(smem + kOffK + s * kTileBytes + h * kHalf, &tmK, &bars[kBarKFull + s], h * 64,
                    c1, c2);
      }
      counts[0] = j + 1;
    }
  } else if (warp == 2 && lane == 0) {
    // ---- V producer ----
    prefetch_tensormap(&tmV);
    for (int j = 0; j < n_tiles; ++j) {
      const int s = j % kStages;
      if (j >= kStages && !wait_bar(&bars[kBarVEmpty + s], ((j / kStages) - 1) & 1, abort_flag)) break;
      mbar_arrive_expect_tx(&bars[kBarVFull + s], kTileBytes);
      for (int h = 0; h < 2; ++h) {
        const int t = j * kBN;
        const int c1 = p.kv_tok_coord == 1 ? t : kvh, c2 = p.kv_tok_coord == 1 ? kvh : t;
        tma_load_3d(smem + kOffV + s * kTileBytes + h * kHalf, &tmV, &bars[kBarVFull + s], h * 64,
                    c1, c2);
      }
      counts[1] = j + 1;
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    auto issue_pv = [&](int i) -> bool {
      if (!wait_bar(&bars[kBarPFull], i & 1, abort_flag)) return false;
      const int s = i % kStages;
      if (!wait_bar(&bars[kBarVFull + s], (i / kStages) & 1, abort_flag)) return false;
      tc_fence_after();
      const uint32_t vb = sbase + kOffV + s * kTileBytes;
#pragma unroll
      for (int k = 0; k < kBN / 16; ++k) {
        // P_i in TMEM over S[i&1]: 16 keys = 8 packed columns. V: MN-major (dims contiguous),
        // 16 keys = two 8-row groups (2 x 1024 B); the 64-dim halves are 16 KB apart.
        const uint64_t db = smem_desc(vb + k * 2048, kHalf, 1024);
        mma_f16_ts(tO, tS[i & 1] + k * 8, db, kIdescPV, (i > 0 || k > 0) ? 1u : 0u);
      }
      mma_commit(&bars[kBarVEmpty + s]);
      mma_commit(&bars[kBarPVDone]);
      counts[3] = i + 1;
      return true;
    };
    bool ok = wait_bar(&bars[kBarQ], 0, abort_flag);
    for (int j = 0; ok && j < n_tiles; ++j) {
      const int s = j % kStages, b = j & 1;
      if (!wait_bar(&bars[kBarKFull + s], (j / kStages) & 1, abort_flag)) break;
      // S[b] still holds P_{j-2}; PV_{j-2} was issued before this point, and MMAs run in order.
      tc_fence_after();
      const uint32_t qa = sbase + kOffQ, kb = sbase + kOffK + s * kTileBytes;
#pragma unroll
      for (int k = 0; k < kHD / 16; ++k) {
        const uint64_t da = smem_desc(qa + (k >> 2) * kHalf + (k & 3) * 32, 16, 1024);
        const uint64_t db = smem_desc(kb + (k >> 2) * kHalf + (k & 3) * 32, 16, 1024);
        mma_f16(tS[b], da, db, kIdescQK, k > 0 ? 1u : 0u);
      }
      mma_commit(&bars[kBarSFull + b]);
      mma_commit(&bars[kBarKEmpty + s]);
      counts[2] = j + 1;
      if (j >= 1 && !issue_pv(j - 1)) {
        ok = false;
        break;
      }
    }
    if (ok && n_tiles > 0) issue_pv(n_tiles - 1);
  } else if (warp >= 4) {
    // ---- softmax: group g, thread r owns query row r, key columns [64g, 64g+64) ----
    const int g = (warp - 4) >> 2;                 // 0 or 1
    const int r = (tid - 128) & 127;               // TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(((warp - 4) & 3) * 32) << 16;
    const int qi = q0 + r;                         // query index within the prompt
    const int row_limit = offset + qi;             // last visible key (causal)
    float* xmax = reinterpret_cast<float*>(smem + kOffX);  // [parity][group][row]
    float* xsum = xmax + 2 * 2 * kBM;                       // [group][row]
    float m_used = -INFINITY, l_sum = 0.f;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int b = j & 1;
      if (!__all_sync(0xffffffffu, wait_bar(&bars[kBarSFull + b], (j >> 1) & 1, abort_flag))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sv[64];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float v[32];
        tmem_ld32(tS[b] + lane_off + 64 * g + c * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) sv[c * 32 + i] = v[i];
      }
      // Raw-score maxima (the scale is positive, so it commutes with max); keys past the causal
      // limit or the sequence end are -inf. Only diagonal / partial tiles need the mask.
      const bool need_mask =
          (p.causal && j * kBN + kBN - 1 > offset + q0) || (j * kBN + kBN > p.kv_len);
      if (need_mask) {
        // keys j*128 + 64g + i with i >= nv are past the sequence or above the causal limit
        const int lim = p.causal ? min(p.kv_len, row_limit + 1) : p.kv_len;
        const int nv = lim - (j * kBN + 64 * g);
#pragma unroll
        for (int i = 0; i < 64; ++i) sv[i] = i < nv ? sv[i] : -INFINITY;
      }
      float mx8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx8[i] = sv[i];
#pragma unroll
      for (int i = 8; i < 64; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], sv[i]);
      float pmax = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                         fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      // exchange partial maxima with the other group (double-buffered by tile parity): only the
      // two warps that hold these 32 rows (warp 4+w of group 0, 8+w of group 1) meet here
      xmax[(b * 2 + g) * kBM + r] = pmax;
      const int xbar = kBarXMax + b * 4 + ((warp - 4) & 3);
      mbar_arrive(&bars[xbar]);
      if (!__all_sync(0xffffffffu, wait_bar(&bars[xbar], (j >> 1) & 1, abort_flag))) {
        ok = false;
        break;
      }
      const float row_max = fmaxf(pmax, xmax[(b * 2 + (g ^ 1)) * kBM + r]) * p.scale_log2;
      const float m_new = fmaxf(m_used, row_max);
      const bool grow = m_used == -INFINITY || m_new > m_used + kRescaleLog2;
      if (__any_sync(0xffffffffu, grow && j > 0)) {
        // Rescale this warp's rows of O (our 64 columns) once PV_{j-1} has landed.
        if (!__all_sync(0xffffffffu, wait_bar(&bars[kBarPVDone], (j - 1) & 1, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float alpha =
            (m_used == -INFINITY || m_new == -INFINITY) ? 1.f : ex2(m_used - m_new);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float v[32];
          tmem_ld32(tO + lane_off + 64 * g + c * 32, v);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] *= alpha;
          tmem_st32(tO + lane_off + 64 * g + c * 32, v);
        }
        tmem_wait_st();
        l_sum *= alpha;
        m_used = m_new;
      } else if (grow) {
        m_used = m_new;  // first tile: nothing accumulated yet
      }
      const float ref = m_used == -INFINITY ? 0.f : m_used;
      // p = 2^(s * scale_log2 - ref): one packed FMA per pair, then the exp, sum and bf16 pack.
      const uint64_t scale2 = f2_pack(p.scale_log2, p.scale_log2);
      const uint64_t nref2 = f2_pack(-ref, -ref);
      uint64_t sum2[4] = {0ull, 0ull, 0ull, 0ull};
      uint32_t pk[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        float x0, x1;
        f2_unpack(f2_fma(f2_pack(sv[2 * i], sv[2 * i + 1]), scale2, nref2), x0, x1);
        const float a0 = ex2(x0), a1 = ex2(x1);
        sum2[i & 3] = f2_add(sum2[i & 3], f2_pack(a0, a1));
        pk[i] = pack_bf16x2(a0, a1);
      }
      {
        float s0, s1;
        f2_unpack(f2_add(f2_add(sum2[0], sum2[1]), f2_add(sum2[2], sum2[3])), s0, s1);
        l_sum += s0 + s1;
      }
      // P slice over S: keys [64g, 64g+64) = packed columns [32g, 32g+32) of buffer b
      tmem_st32u(tS[b] + lane_off + 32 * g, pk);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars[kBarPFull]);
    }
    if (ok && n_tiles > 0 &&
        __all_sync(0xffffffffu, wait_bar(&bars[kBarPVDone], (n_tiles - 1) & 1, abort_flag))) {
      tc_fence_after();
      xsum[g * kBM + r] = l_sum;
      mbar_arrive(&bars[kBarXSum]);
      if (__all_sync(0xffffffffu, wait_bar(&bars[kBarXSum], 0, abort_flag))) {
        const float total = l_sum + xsum[(g ^ 1) * kBM + r];
        const float inv = total > 0.f ? 1.f / total : 0.f;
        // The normalised tile goes through shared memory (the K ring, idle once every MMA is done;
        // rows padded to kStageRow bytes so a warp's 32 rows fall in distinct bank groups), then
        // out in whole rows: a thread's own row is 8 KB from its neighbour's, so direct stores
        // would touch 32 half sectors per instruction (1.2 us of the epilogue).
        uint8_t* stage = smem + kOffK;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float v[32];
          tmem_ld32(tO + lane_off + 64 * g + c * 32, v);
          tmem_wait_ld();
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8) {
            uint4 o4;
            o4.x = pack_bf16x2(v[q8 * 8 + 0] * inv, v[q8 * 8 + 1] * inv);
            o4.y = pack_bf16x2(v[q8 * 8 + 2] * inv, v[q8 * 8 + 3] * inv);
            o4.z = pack_bf16x2(v[q8 * 8 + 4] * inv, v[q8 * 8 + 5] * inv);
            o4.w = pack_bf16x2(v[q8 * 8 + 6] * inv, v[q8 * 8 + 7] * inv);
            *reinterpret_cast<uint4*>(stage + r * kStageRow + g * 128 + c * 64 + q8 * 16) = o4;
          }
        }
        mbar_arrive(&bars[kBarOStaged]);
        if (__all_sync(0xffffffffu, wait_bar(&bars[kBarOStaged], 0, abort_flag))) {
          for (int i = tid - 128; i < kBM * 16; i += kSoftmaxThreads) {
            const int row = i >> 4, ch = i & 15;
            if (q0 + row < p.q_len)
              *reinterpret_cast<uint4*>(p.out + static_cast<int64_t>(q0 + row) * p.o_st +
                                        static_cast<int64_t>(head) * p.o_sh + ch * 8) =
                  *reinterpret_cast<const uint4*>(stage + row * kStageRow + ch * 16);
          }
        }
      }
    }
  }

  // ---- teardown: everyone meets here; on abort, let in-flight async work land first ----
  tc_fence_before();
  __syncthreads();
  if (*abort_flag && tid == 0) {
    // Let every copy and MMA still in flight land before the CTA releases its shared memory and
    // TMEM: the newest fill of each stage, the Q fill, and the last QK and PV commits (commits
    // complete in order, so the last one covers every MMA before it). Bounded like every wait.
    const unsigned long long t0 = globaltimer_ns();
    auto drain = [&](uint64_t* bar, uint32_t parity) {
      while (!mbar_try_wait(smem_u32(bar), parity) && globaltimer_ns() - t0 < kWaitLimitNs) {
      }
    };
    drain(&bars[kBarQ], 0);
    for (int t = max(0, counts[0] - kStages); t < counts[0]; ++t)
      drain(&bars[kBarKFull + t % kStages], (t / kStages) & 1);
    for (int t = max(0, counts[1] - kStages); t < counts[1]; ++t)
      drain(&bars[kBarVFull + t % kStages], (t / kStages) & 1);
    if (counts[2] > 0) drain(&bars[kBarSFull + ((counts[2] - 1) & 1)], ((counts[2] - 1) >> 1) & 1);
    if (counts[3] > 0) drain(&bars[kBarPVDone], (counts[3] - 1) & 1);
  }
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();  // lane 0 ran the MMA role alone: reconverge for the warp-collective dealloc
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols));
  }
}

// ------------------------------------------------------------------------------------------
// Persistent variant for grids with more (query tile, head) items than SMs: at most one CTA per
// SM, each walking its list of items (item_of below) with the one-tile kernel's roles and math.
// The roles keep running counts over items: the K/V rings and the S/P buffers continue across
// item boundaries; Q and O are double-buffered by item parity, so the next item's Q tile, first
// K/V tiles and first QK run while the current item finishes. The epilogue of item k (normalise
// and store) runs after item k + 1's first P is written, with the tensor core busy on that
// item's MMAs, and stages the output tile in item k's Q buffer. One item per CTA stays on
// prefill_kernel: with nothing to overlap, this variant measured 0.6-0.7 us slower per call.
namespace items {

constexpr int kStageRow = kHD * 2;  // bytes per staged output row (16-byte chunks XOR-swizzled)

// shared memory map (offsets from a 1024-aligned base). Q is double-buffered by item parity; once
// an item's MMAs are done its Q buffer holds the item's normalised output tile for the store.
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + 2 * kTileBytes;
constexpr int kOffV = kOffK + kStages * kTileBytes;
constexpr int kOffX = kOffV + kStages * kTileBytes;  // row-max exchange [2][2][128] + sums [2][128]
constexpr int kOffBar = kOffX + 3 * 2 * kBM * 4;
constexpr int kSmemBytes = 1024 + kOffBar + 512;

// Barrier indices. "Item parity" is the parity of the item's ordinal within its CTA; "tile" is
// the CTA's running count of K/V tiles over all its items.
enum {
  kBarQFull = 0,                     // +item parity: Q tile landed
  kBarQEmpty = kBarQFull + 2,        // +item parity, 256 arrivals: the staged output read back,
                                     // buffer free (arrived only if item k + 2 exists)
  kBarKFull = kBarQEmpty + 2,        // +stage
  kBarKEmpty = kBarKFull + kStages,
  kBarVFull = kBarKEmpty + kStages,
  kBarVEmpty = kBarVFull + kStages,
  kBarSFull = kBarVEmpty + kStages,  // +buffer (2): QK of a tile committed
  kBarPFull = kBarSFull + 2,         // 256 arrivals: P of a tile written to TMEM
  kBarPVDone = kBarPFull + 1,        // PV of a tile committed
  kBarOFull = kBarPVDone + 1,        // +item parity: the item's last PV committed
  kBarXMax = kBarOFull + 2,          // +parity*4 + warp pair (8), 64 arrivals: row-max exchange
  kBarXSum = kBarXMax + 8,           // 256 arrivals: final row-sum exchange
  kBarOStaged = kBarXSum + 1,        // 256 arrivals: the output tile staged in shared memory
  kNumBars = kBarOStaged + 1
};

// Work items: (128-row query tile, query head) pairs, heaviest query tiles first (item w = query
// tile q_tiles - 1 - w / nh of head w % nh). CTA c of a grid of G takes items c, 2G - 1 - c,
// 2G + c, 4G - 1 - c, ...: a snake over the grid that gives the CTAs holding the heaviest first
// items the lightest second ones.
__device__ __forceinline__ int item_of(int k, int c, int grid) {
  return k * grid + ((k & 1) ? grid - 1 - c : c);
}

struct Item {
  int q0, head, kvh, n_tiles;
};

__device__ __forceinline__ Item item_info(int w, const Params& p) {
  Item it;
  it.q0 = (p.q_tiles - 1 - w / p.nh) * kBM;
  it.head = w % p.nh;
  it.kvh = it.head / p.group;
  const int kv_tiles_all = (p.kv_len + kBN - 1) / kBN;
  it.n_tiles = kv_tiles_all;
  if (p.causal) {
    const int last_row = min(it.q0 + kBM, p.q_len) - 1;
    const int last_key = p.kv_len - p.q_len + last_row;  // >= 0: the host requires q_len <= kv_len
    it.n_tiles = min(kv_tiles_all, last_key / kBN + 1);
  }
  // kv_len >= 1 and (causal) q_len <= kv_len make every item see at least one key; the clamp only
  // keeps the roles' per-item barrier counts in step should that ever change.
  it.n_tiles = max(it.n_tiles, 1);
  return it;
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    prefill_items_kernel(const __grid_constant__ CUtensorMap tmQ,
                         const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // issue / commit counts, read by the abort drain: [0] K tiles, [1] V tiles, [2] QK, [3] PV,
  // [4] Q tiles
  volatile int* counts = reinterpret_cast<volatile int*>(tmem_slot + 2);
  const uint32_t sbase = smem_u32(smem);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int cta = static_cast<int>(blockIdx.x), grid = static_cast<int>(gridDim.x);
  const int n_items = p.q_tiles * p.nh;

  if (tid == 0) {
    for (int i = 0; i < kNumBars; ++i) {
      const uint32_t count =
          (i == kBarPFull || i == kBarXSum || i == kBarOStaged || i == kBarQEmpty ||
           i == kBarQEmpty + 1)
              ? kSoftmaxThreads
          : (i >= kBarXMax && i < kBarXMax + 8) ? 64u
                                                 : 1u;
      mbar_init(&bars[i], count);
    }
    *abort_flag = 0;
    for (int i = 0; i < 5; ++i) counts[i] = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Launched as a programmatic dependent: everything above (barriers, TMEM) overlaps the previous
  // kernel's tail; Q, K, V and the output are touched only after it has finished. The next kernel
  // may launch only now, once every CTA holds its TMEM: a dependent CTA that took the columns
  // first would wait on this grid while this CTA waited on the columns.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  // TMEM columns: S/P double buffer by tile parity, O double buffer by item parity
  auto tS = [&](int b) -> uint32_t { return tmem + static_cast<uint32_t>(b & 1) * kBN; };
  auto tO = [&](int k) -> uint32_t { return tmem + static_cast<uint32_t>(2 + (k & 1)) * kBN; };

  if (warp == 3 && lane == 0) {
    // ---- Q producer: one tile per item into the buffer of the item's parity ----
    prefetch_tensormap(&tmQ);
    for (int k = 0;; ++k) {
      const int w = item_of(k, cta, grid);
      if (w >= n_items) break;
      const Item it = item_info(w, p);
      const int qb = k & 1;
      // One Q tile in flight at a time: the first item's Q and K tiles go out first.
      if (k >= 1 && !wait_bar(&bars[kBarQFull + (qb ^ 1)], ((k - 1) >> 1) & 1, abort_flag)) break;
      if (k >= 2 && !wait_bar(&bars[kBarQEmpty + qb], ((k >> 1) - 1) & 1, abort_flag)) break;
      mbar_arrive_expect_tx(&bars[kBarQFull + qb], kTileBytes);
      for (int h = 0; h < 2; ++h) {
        const int c1 = p.q_tok_coord == 1 ? it.q0 : it.head, c2 = p.q_tok_coord == 1 ? it.head : it.q0;
        tma_load_3d(smem + kOffQ + qb * kTileBytes + h * kHalf, &tmQ, &bars[kBarQFull + qb], h * 64,
                    c1, c2);
      }
      counts[4] = k + 1;
    }
  } else if (warp == 0 || warp == 2) {
    // ---- K (warp 0) and V (warp 2) producers: one ring each over the CTA's items ----
    if (lane == 0) {
      const bool is_k = warp == 0;
      const CUtensorMap* tm = is_k ? &tmK : &tmV;
      const int full = is_k ? kBarKFull : kBarVFull, empty = is_k ? kBarKEmpty : kBarVEmpty;
      uint8_t* ring = smem + (is_k ? kOffK : kOffV);
      prefetch_tensormap(tm);
      int gt = 0;
      // V tiles are needed one softmax later than K tiles: let the first K tile go out first.
      bool ok = is_k || wait_bar(&bars[kBarKFull], 0, abort_flag);
      for (int k = 0; ok; ++k) {
        const int w = item_of(k, cta, grid);
        if (w >= n_items) break;
        const Item it = item_info(w, p);
        for (int j = 0; j < it.n_tiles; ++j, ++gt) {
          const int s = gt % kStages;
          if (gt >= kStages && !wait_bar(&bars[empty + s], ((gt / kStages) - 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&bars[full + s], kTileBytes);
          for (int h = 0; h < 2; ++h) {
            const int t = j * kBN;
            const int c1 = p.kv_tok_coord == 1 ? t : it.kvh, c2 = p.kv_tok_coord == 1 ? it.kvh : t;
            tma_load_3d(ring + s * kTileBytes + h * kHalf, tm, &bars[full + s], h * 64, c1, c2);
          }
          counts[is_k ? 0 : 1] = gt + 1;
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer: one stream of tiles over the CTA's items; PV of a tile is issued after the
    // QK of the next one (the next item's first QK included), so S is ready before it is needed.
    auto issue_pv = [&](int g, int j, int k, bool last) -> bool {
      if (!wait_bar(&bars[kBarPFull], g & 1, abort_flag)) return false;
      const int s = g % kStages;
      if (!wait_bar(&bars[kBarVFull + s], (g / kStages) & 1, abort_flag)) return false;
      tc_fence_after();
      const uint32_t vb = sbase + kOffV + s * kTileBytes;
#pragma unroll
      for (int kk = 0; kk < kBN / 16; ++kk) {
        // P over S[g&1]: 16 keys = 8 packed columns. V: MN-major (dims contiguous), 16 keys =
        // two 8-row groups (2 x 1024 B); the 64-dim halves are 16 KB apart.
        const uint64_t db = smem_desc(vb + kk * 2048, kHalf, 1024);
        mma_f16_ts(tO(k & 1), tS(g & 1) + kk * 8, db, kIdescPV, (j > 0 || kk > 0) ? 1u : 0u);
      }
      mma_commit(&bars[kBarVEmpty + s]);
      mma_commit(&bars[kBarPVDone]);
      if (last) mma_commit(&bars[kBarOFull + (k & 1)]);
      counts[3] = g + 1;
      return true;
    };
    int gt = 0, pend_g = -1, pend_j = 0, pend_k = 0;
    bool pend_last = false, ok = true;
    for (int k = 0; ok; ++k) {
      const int w = item_of(k, cta, grid);
      if (w >= n_items) break;
      const Item it = item_info(w, p);
      if (!wait_bar(&bars[kBarQFull + (k & 1)], (k >> 1) & 1, abort_flag)) {
        ok = false;
        break;
      }
      const uint32_t qa = sbase + kOffQ + (k & 1) * kTileBytes;
      for (int j = 0; j < it.n_tiles; ++j, ++gt) {
        const int s = gt % kStages, b = gt & 1;
        if (!wait_bar(&bars[kBarKFull + s], (gt / kStages) & 1, abort_flag)) {
          ok = false;
          break;
        }
        // S[b] still holds P of tile gt-2; its PV was issued before this point, and MMAs run in
        // issue order.
        tc_fence_after();
        const uint32_t kb = sbase + kOffK + s * kTileBytes;
#pragma unroll
        for (int kk = 0; kk < kHD / 16; ++kk) {
          const uint64_t da = smem_desc(qa + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
          const uint64_t db = smem_desc(kb + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
          mma_f16(tS(b), da, db, kIdescQK, kk > 0 ? 1u : 0u);
        }
        mma_commit(&bars[kBarSFull + b]);
        mma_commit(&bars[kBarKEmpty + s]);
        counts[2] = gt + 1;
        if (pend_g >= 0 && !issue_pv(pend_g, pend_j, pend_k, pend_last)) {
          ok = false;
          break;
        }
        pend_g = gt;
        pend_j = j;
        pend_k = k;
        pend_last = j == it.n_tiles - 1;
      }
    }
    if (ok && pend_g >= 0) issue_pv(pend_g, pend_j, pend_k, pend_last);
  } else if (warp >= 4) {
    // ---- softmax: group g, thread r owns query row r, key columns [64g, 64g+64) ----
    const int g = (warp - 4) >> 2;                 // 0 or 1
    const int r = (tid - 128) & 127;               // TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(((warp - 4) & 3) * 32) << 16;
    const int offset = p.kv_len - p.q_len;         // bottom-right alignment
    float* xmax = reinterpret_cast<float*>(smem + kOffX);  // [parity][group][row]
    float* xsum = xmax + 2 * 2 * kBM;                       // [group][row]
    // Normalise and store item k's output. Runs after the next item's first P is written (or
    // after the last item), so the tensor core already has that item's PV and next QK queued.
    auto epilogue = [&](int k, float l_item) -> bool {
      const Item ie = item_info(item_of(k, cta, grid), p);
      const int q0 = ie.q0, head = ie.head;
      if (!__all_sync(0xffffffffu, wait_bar(&bars[kBarOFull + (k & 1)], (k >> 1) & 1, abort_flag)))
        return false;
      tc_fence_after();
      xsum[g * kBM + r] = l_item;
      mbar_arrive(&bars[kBarXSum]);
      if (!__all_sync(0xffffffffu, wait_bar(&bars[kBarXSum], k & 1, abort_flag))) return false;
      const float total = l_item + xsum[(g ^ 1) * kBM + r];
      const float inv = total > 0.f ? 1.f / total : 0.f;
      // The normalised tile goes through the item's Q buffer (its QK MMAs are complete: they were
      // issued before the item's last PV), 16-byte chunk c of row r at chunk c ^ (r & 15) so a
      // warp's 32 rows fall in distinct bank groups, then out in whole rows: a thread's own row
      // is 8 KB from its neighbour's, so direct stores would touch 32 half sectors per instruction.
      uint8_t* stage = smem + kOffQ + (k & 1) * kTileBytes;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float v[16];
        tmem_ld16(tO(k & 1) + lane_off + 64 * g + c * 16, v);
        tmem_wait_ld();
#pragma unroll
        for (int q8 = 0; q8 < 2; ++q8) {
          uint4 o4;
          o4.x = pack_bf16x2(v[q8 * 8 + 0] * inv, v[q8 * 8 + 1] * inv);
          o4.y = pack_bf16x2(v[q8 * 8 + 2] * inv, v[q8 * 8 + 3] * inv);
          o4.z = pack_bf16x2(v[q8 * 8 + 4] * inv, v[q8 * 8 + 5] * inv);
          o4.w = pack_bf16x2(v[q8 * 8 + 6] * inv, v[q8 * 8 + 7] * inv);
          const int chunk = g * 8 + c * 2 + q8;
          *reinterpret_cast<uint4*>(stage + r * kStageRow + ((chunk ^ (r & 15)) << 4)) = o4;
        }
      }
      mbar_arrive(&bars[kBarOStaged]);
      if (!__all_sync(0xffffffffu, wait_bar(&bars[kBarOStaged], k & 1, abort_flag))) return false;
      // Read the whole staged tile first, hand the buffer back (its next writer is the TMA load
      // of item k + 2's Q tile, if the CTA has one), then store.
      constexpr int kPerThread = kBM * 16 / kSoftmaxThreads;
      uint4 o[kPerThread];
#pragma unroll
      for (int t = 0; t < kPerThread; ++t) {
        const int i = tid - 128 + t * kSoftmaxThreads, row = i >> 4, ch = i & 15;
        o[t] = *reinterpret_cast<const uint4*>(stage + row * kStageRow + ((ch ^ (row & 15)) << 4));
      }
      if (item_of(k + 2, cta, grid) < n_items) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive(&bars[kBarQEmpty + (k & 1)]);
      }
#pragma unroll
      for (int t = 0; t < kPerThread; ++t) {
        const int i = tid - 128 + t * kSoftmaxThreads, row = i >> 4, ch = i & 15;
        if (q0 + row < p.q_len)
          *reinterpret_cast<uint4*>(p.out + static_cast<int64_t>(q0 + row) * p.o_st +
                                    static_cast<int64_t>(head) * p.o_sh + ch * 8) = o[t];
      }
      return true;
    };
    int gt = 0, prev_k = -1;
    float prev_l = 0.f;
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int w = item_of(k, cta, grid);
      const bool have = w < n_items;
      if (!have && prev_k < 0) break;
      const Item it = item_info(have ? w : 0, p);
      const int row_limit = offset + it.q0 + r;    // last visible key (causal)
      float m_used = -INFINITY, l_sum = 0.f;
      // Past the last item one more pass runs only the deferred epilogue (one call site).
      const int n_pass = have ? it.n_tiles : 1;
      for (int j = 0; j < n_pass; ++j) {
       if (have) {
        const int b = gt & 1;
        if (!__all_sync(0xffffffffu, wait_bar(&bars[kBarSFull + b], (gt >> 1) & 1, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
        float sv[64];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float v[32];
          tmem_ld32(tS(b) + lane_off + 64 * g + c * 32, v);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) sv[c * 32 + i] = v[i];
        }
        // Raw-score maxima (the scale is positive, so it commutes with max); keys past the causal
        // limit or the sequence end are -inf. Only diagonal / partial tiles need the mask.
        const bool need_mask =
            (p.causal && j * kBN + kBN - 1 > offset + it.q0) || (j * kBN + kBN > p.kv_len);
        if (need_mask) {
          // keys j*128 + 64g + i with i >= nv are past the sequence or above the causal limit
          const int lim = p.causal ? min(p.kv_len, row_limit + 1) : p.kv_len;
          const int nv = lim - (j * kBN + 64 * g);
#pragma unroll
          for (int i = 0; i < 64; ++i) sv[i] = i < nv ? sv[i] : -INFINITY;
        }
        float mx8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mx8[i] = sv[i];
#pragma unroll
        for (int i = 8; i < 64; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], sv[i]);
        float pmax = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                           fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
        // exchange partial maxima with the other group (double-buffered by tile parity): only the
        // two warps that hold these 32 rows (warp 4+w of group 0, 8+w of group 1) meet here
        xmax[(b * 2 + g) * kBM + r] = pmax;
        const int xbar = kBarXMax + b * 4 + ((warp - 4) & 3);
        mbar_arrive(&bars[xbar]);
        if (!__all_sync(0xffffffffu, wait_bar(&bars[xbar], (gt >> 1) & 1, abort_flag))) {
          ok = false;
          break;
        }
        const float row_max = fmaxf(pmax, xmax[(b * 2 + (g ^ 1)) * kBM + r]) * p.scale_log2;
        const float m_new = fmaxf(m_used, row_max);
        const bool grow = m_used == -INFINITY || m_new > m_used + kRescaleLog2;
        if (__any_sync(0xffffffffu, grow && j > 0)) {
          // Rescale this warp's rows of O (our 64 columns) once the previous tile's PV has landed
          // (QK of this tile was issued after the PV before it, so that one is the newest).
          if (!__all_sync(0xffffffffu, wait_bar(&bars[kBarPVDone], (gt - 1) & 1, abort_flag))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const float alpha =
              (m_used == -INFINITY || m_new == -INFINITY) ? 1.f : ex2(m_used - m_new);
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            float v[16];
            tmem_ld16(tO(k & 1) + lane_off + 64 * g + c * 16, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] *= alpha;
            tmem_st16(tO(k & 1) + lane_off + 64 * g + c * 16, v);
          }
          tmem_wait_st();
          l_sum *= alpha;
          m_used = m_new;
        } else if (grow) {
          m_used = m_new;  // first tile: nothing accumulated yet
        }
        const float ref = m_used == -INFINITY ? 0.f : m_used;
        // p = 2^(s * scale_log2 - ref): one packed FMA per pair, then the exp, sum and bf16 pack.
        const uint64_t scale2 = f2_pack(p.scale_log2, p.scale_log2);
        const uint64_t nref2 = f2_pack(-ref, -ref);
        uint64_t sum2[4] = {0ull, 0ull, 0ull, 0ull};
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float x0, x1;
          f2_unpack(f2_fma(f2_pack(sv[2 * i], sv[2 * i + 1]), scale2, nref2), x0, x1);
          const float a0 = ex2(x0), a1 = ex2(x1);
          sum2[i & 3] = f2_add(sum2[i & 3], f2_pack(a0, a1));
          pk[i] = pack_bf16x2(a0, a1);
        }
        {
          float s0, s1;
          f2_unpack(f2_add(f2_add(sum2[0], sum2[1]), f2_add(sum2[2], sum2[3])), s0, s1);
          l_sum += s0 + s1;
        }
        // P slice over S: keys [64g, 64g+64) = packed columns [32g, 32g+32) of buffer b
        tmem_st32u(tS(b) + lane_off + 32 * g, pk);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&bars[kBarPFull]);
        ++gt;
       }
        if (j == 0 && prev_k >= 0) {
          if (!epilogue(prev_k, prev_l)) {
            ok = false;
            break;
          }
        }
      }
      if (!have) break;
      prev_k = k;
      prev_l = l_sum;
    }
  }

  // ---- teardown: everyone meets here; on abort, let in-flight async work land first ----
  tc_fence_before();
  __syncthreads();
  if (*abort_flag && tid == 0) {
    // Let every copy and MMA still in flight land before the CTA releases its shared memory and
    // TMEM: the newest fill of each stage and Q buffer, and the last QK and PV commits (commits
    // complete in order, so the last one covers every MMA before it). Bounded like every wait.
    const unsigned long long t0 = globaltimer_ns();
    auto drain = [&](uint64_t* bar, uint32_t parity) {
      while (!mbar_try_wait(smem_u32(bar), parity) && globaltimer_ns() - t0 < kWaitLimitNs) {
      }
    };
    for (int t = max(0, counts[4] - 2); t < counts[4]; ++t)
      drain(&bars[kBarQFull + (t & 1)], (t >> 1) & 1);
    for (int t = max(0, counts[0] - kStages); t < counts[0]; ++t)
      drain(&bars[kBarKFull + t % kStages], (t / kStages) & 1);
    for (int t = max(0, counts[1] - kStages); t < counts[1]; ++t)
      drain(&bars[kBarVFull + t % kStages], (t / kStages) & 1);
    if (counts[2] > 0) drain(&bars[kBarSFull + ((counts[2] - 1) & 1)], ((counts[2] - 1) >> 1) & 1);
    if (counts[3] > 0) drain(&bars[kBarPVDone], (counts[3] - 1) & 1);
  }
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();  // lane 0 ran the MMA role alone: reconverge for the warp-collective dealloc
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols));
  }
}

}  // namespace items
// ------------------------------------------------------------------------------------------
// Ping-pong variant for long prompts: one CTA computes TWO 128-row query tiles (A = rows
// q0..q0+127, B = the next 128) of one head against one stream of K/V tiles. TMEM holds S_A, O_A,
// S_B, O_B (128 columns each); P_x is written over the first 64 columns of S_x. Each tile has its
// own softmax warp group (warps 4-7 for A, 8-11 for B), thread r owning the whole 128-key row r, so
// no values are exchanged between groups. The MMA warp interleaves the tiles:
//   QK_A(0) QK_B(0) | PV_A(j) QK_A(j+1) PV_B(j) QK_B(j+1) | ...
// so while group A turns S_A(j) into P_A(j) the tensor core runs PV_B(j-1) and QK_B(j), and the
// other way round: one tile's MMAs and TMEM load latency hide under the other tile's softmax.
// QK_x(j+1) is issued after PV_x(j) (which reads P_x(j) out of S_x); the MMAs of one CTA run in
// issue order. K/V tiles are shared by both query tiles (half the K/V traffic per query of the
// one-tile kernel). Every wait is bounded; the abort path drains like the one-tile kernel.
namespace pp {

constexpr int kRows = 2 * kBM;                   // query rows per CTA
constexpr int kOffQA = 0;
constexpr int kOffQB = kOffQA + kTileBytes;
constexpr int kOffK = kOffQB + kTileBytes;
constexpr int kOffV = kOffK + kStages * kTileBytes;
constexpr int kOffBar = kOffV + kStages * kTileBytes;
constexpr int kSmemBytes = 1024 + kOffBar + 512;

enum {
  kBarQ = 0,
  kBarKFull = 1,                      // +stage
  kBarKEmpty = kBarKFull + kStages,
  kBarVFull = kBarKEmpty + kStages,
  kBarVEmpty = kBarVFull + kStages,
  kBarSFull = kBarVEmpty + kStages,   // +tile (A, B): QK_x(j) committed
  kBarPFull = kBarSFull + 2,          // +tile, 128 arrivals: P_x(j) in TMEM
  kBarPVDone = kBarPFull + 2,         // +tile: PV_x(j) committed
  kNumBars = kBarPVDone + 2
};

__device__ __forceinline__ void tmem_st8u(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
      : "memory");
}

__device__ __forceinline__ void tmem_st16u(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    prefill_pp_kernel(const __grid_constant__ CUtensorMap tmQ,
                      const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // issue / commit counts for the abort drain: K, V, QK_A, QK_B, PV_A, PV_B
  volatile int* counts = reinterpret_cast<volatile int*>(tmem_slot + 2);
  const uint32_t sbase = smem_u32(smem);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int pair_tiles = (p.q_tiles + 1) / 2;
  const int q_pair = pair_tiles - 1 - static_cast<int>(blockIdx.x) / p.nh;  // heaviest first
  const int head = static_cast<int>(blockIdx.x) % p.nh;
  const int kvh = head / p.group;
  const int q0 = q_pair * kRows;
  const int offset = p.kv_len - p.q_len;  // bottom-right alignment
  const int kv_tiles_all = (p.kv_len + kBN - 1) / kBN;
  int n_t[2];  // KV tiles each query tile needs (0 for a tile past the prompt)
#pragma unroll
  for (int x = 0; x < 2; ++x) {
    const int first = q0 + x * kBM;
    if (first >= p.q_len) {
      n_t[x] = 0;
    } else if (!p.causal) {
      n_t[x] = kv_tiles_all;
    } else {
      const int last_key = offset + min(first + kBM, p.q_len) - 1;
      n_t[x] = min(kv_tiles_all, last_key / kBN + 1);
    }
  }
  const int n = max(n_t[0], n_t[1]);

  if (tid == 0) {
    for (int i = 0; i < kNumBars; ++i)
      mbar_init(&bars[i], (i == kBarPFull || i == kBarPFull + 1) ? static_cast<uint32_t>(kBM) : 1u);
    *abort_flag = 0;
    for (int i = 0; i < 6; ++i) counts[i] = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Launched as a programmatic dependent: everything above (barriers, TMEM) overlaps the previous
  // kernel's tail; Q, K, V and the output are touched only after it has finished. The next kernel
  // may launch only now, once every CTA holds its TMEM: a dependent CTA that took the columns
  // first would wait on this grid while this CTA waited on the columns.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS[2] = {tmem, tmem + 2 * kBN};
  const uint32_t tO[2] = {tmem + kBN, tmem + 3 * kBN};

  if (warp == 0 && lane == 0) {
    // ---- Q (both tiles) + K producer ----
    prefetch_tensormap(&tmQ);
    prefetch_tensormap(&tmK);
    mbar_arrive_expect_tx(&bars[kBarQ], 2 * kTileBytes);
    for (int x = 0; x < 2; ++x)
      for (int h = 0; h < 2; ++h) {
        const int t = q0 + x * kBM;  // rows past the prompt load as zeros and are never stored
        const int c1 = p.q_tok_coord == 1 ? t : head, c2 = p.q_tok_coord == 1 ? head : t;
        tma_load_3d(smem + (x ? kOffQB : kOffQA) + h * kHalf, &tmQ, &bars[kBarQ], h * 64, c1, c2);
      }
    for (int j = 0; j < n; ++j) {
      const int s = j % kStages;
      if (j >= kStages && !wait_bar(&bars[kBarKEmpty + s], ((j / kStages) - 1) & 1, abort_flag)) break;
      mbar_arrive_expect_tx(&bars[kBarKFull + s], kTileBytes);
      for (int h = 0; h < 2; ++h) {
        const int t = j * kBN;
        const int c1 = p.kv_tok_coord == 1 ? t : kvh, c2 = p.kv_tok_coord == 1 ? kvh : t;
        tma_load_3d(smem + kOffK + s * kTileBytes + h * kHalf, &tmK, &bars[kBarKFull + s], h * 64,
                    c1, c2);
      }
      counts[0] = j + 1;
    }
  } else if (warp == 2 && lane == 0) {
    // ---- V producer ----
    prefetch_tensormap(&tmV);
    for (int j = 0; j < n; ++j) {
      const int s = j % kStages;
      if (j >= kStages && !wait_bar(&bars[kBarVEmpty + s], ((j / kStages) - 1) & 1, abort_flag)) break;
      mbar_arrive_expect_tx(&bars[kBarVFull + s], kTileBytes);
      for (int h = 0; h < 2; ++h) {
        const int t = j * kBN;
        const int c1 = p.kv_tok_coord == 1 ? t : kvh, c2 = p.kv_tok_coord == 1 ? kvh : t;
        tma_load_3d(smem + kOffV + s * kTileBytes + h * kHalf, &tmV, &bars[kBarVFull + s], h * 64,
                    c1, c2);
      }
      counts[1] = j + 1;
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    auto issue_qk = [&](int x, int j) {
      const uint32_t qa = sbase + (x ? kOffQB : kOffQA);
      const uint32_t kb = sbase + kOffK + (j % kStages) * kTileBytes;
#pragma unroll
      for (int k = 0; k < kHD / 16; ++k) {
        const uint64_t da = smem_desc(qa + (k >> 2) * kHalf + (k & 3) * 32, 16, 1024);
        const uint64_t db = smem_desc(kb + (k >> 2) * kHalf + (k & 3) * 32, 16, 1024);
        mma_f16(tS[x], da, db, kIdescQK, k > 0 ? 1u : 0u);
      }
      mma_commit(&bars[kBarSFull + x]);
      counts[2 + x] = j + 1;
    };
    auto issue_pv = [&](int x, int j) -> bool {
      if (!wait_bar(&bars[kBarPFull + x], j & 1, abort_flag)) return false;
      tc_fence_after();
      const uint32_t vb = sbase + kOffV + (j % kStages) * kTileBytes;
#pragma unroll
      for (int k = 0; k < kBN / 16; ++k) {
        const uint64_t db = smem_desc(vb + k * 2048, kHalf, 1024);
        mma_f16_ts(tO[x], tS[x] + k * 8, db, kIdescPV, (j > 0 || k > 0) ? 1u : 0u);
      }
      mma_commit(&bars[kBarPVDone + x]);
      counts[4 + x] = j + 1;
      return true;
    };
    bool ok = wait_bar(&bars[kBarQ], 0, abort_flag);
    if (ok && n > 0) {
      ok = wait_bar(&bars[kBarKFull], 0, abort_flag);
      if (ok) {
        tc_fence_after();
        if (n_t[0] > 0) issue_qk(0, 0);
        if (n_t[1] > 0) issue_qk(1, 0);
        mma_commit(&bars[kBarKEmpty]);
      }
    }
    for (int j = 0; ok && j < n; ++j) {
      const int s = j % kStages;
      if (!wait_bar(&bars[kBarVFull + s], (j / kStages) & 1, abort_flag)) break;
      tc_fence_after();
      if (j < n_t[0] && !issue_pv(0, j)) break;
      const bool next = j + 1 < n;
      if (next) {
        const int s1 = (j + 1) % kStages;
        if (!wait_bar(&bars[kBarKFull + s1], ((j + 1) / kStages) & 1, abort_flag)) break;
        tc_fence_after();
      }
      if (j + 1 < n_t[0]) issue_qk(0, j + 1);
      if (j < n_t[1] && !issue_pv(1, j)) break;
      mma_commit(&bars[kBarVEmpty + s]);
      if (j + 1 < n_t[1]) issue_qk(1, j + 1);
      if (next) mma_commit(&bars[kBarKEmpty + (j + 1) % kStages]);
    }
  } else if (warp >= 4) {
    // ---- softmax: group x owns query tile x; thread r owns its whole 128-key row r ----
    const int x = (warp - 4) >> 2;
    const int r = (tid - 128) & 127;
    const uint32_t lane_off = static_cast<uint32_t>(((warp - 4) & 3) * 32) << 16;
    const int qi = q0 + x * kBM + r;
    const int row_limit = offset + qi;
    const int nx = n_t[x];
    float m_used = -INFINITY, l_sum = 0.f;
    bool ok = true;
    for (int j = 0; j < nx; ++j) {
      if (!__all_sync(0xffffffffu, wait_bar(&bars[kBarSFull + x], j & 1, abort_flag))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sv[128];
      tmem_ld32(tS[x] + lane_off, *reinterpret_cast<float(*)[32]>(sv));
      tmem_ld32(tS[x] + lane_off + 32, *reinterpret_cast<float(*)[32]>(sv + 32));
      tmem_ld32(tS[x] + lane_off + 64, *reinterpret_cast<float(*)[32]>(sv + 64));
      tmem_ld32(tS[x] + lane_off + 96, *reinterpret_cast<float(*)[32]>(sv + 96));
      tmem_wait_ld();
      const bool need_mask =
          (p.causal && j * kBN + kBN - 1 > offset + q0 + x * kBM) || (j * kBN + kBN > p.kv_len);
      if (need_mask) {
        // keys j*128 + i with i >= nv are past the sequence or above the causal limit
        const int lim = p.causal ? min(p.kv_len, row_limit + 1) : p.kv_len;
        const int nv = lim - j * kBN;
#pragma unroll
        for (int i = 0; i < 128; ++i) sv[i] = i < nv ? sv[i] : -INFINITY;
      }
      float mx8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx8[i] = sv[i];
#pragma unroll
      for (int i = 8; i < 128; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], sv[i]);
      const float row_max = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                                  fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]))) *
                            p.scale_log2;
      const float m_new = fmaxf(m_used, row_max);
      const bool grow = m_used == -INFINITY || m_new > m_used + kRescaleLog2;
      const float alpha =
          (grow && j > 0 && m_used != -INFINITY && m_new != -INFINITY) ? ex2(m_used - m_new) : 1.f;
      if (grow) m_used = m_new;
      const float ref = m_used == -INFINITY ? 0.f : m_used;
      // P = 2^(s * scale_log2 - ref), written as packed bf16 over S in 8-column pieces (few live
      // registers beside the 128 scores).
      const uint64_t scale2 = f2_pack(p.scale_log2, p.scale_log2);
      const uint64_t nref2 = f2_pack(-ref, -ref);
      uint64_t sum2[2] = {0ull, 0ull};
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t pk[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int e = c * 16 + 2 * i;
          float x0, x1;
          f2_unpack(f2_fma(f2_pack(sv[e], sv[e + 1]), scale2, nref2), x0, x1);
          const float a0 = ex2(x0), a1 = ex2(x1);
          sum2[i & 1] = f2_add(sum2[i & 1], f2_pack(a0, a1));
          pk[i] = pack_bf16x2(a0, a1);
        }
        tmem_st8u(tS[x] + lane_off + c * 8, pk);
      }
      {
        float s0, s1;
        f2_unpack(f2_add(sum2[0], sum2[1]), s0, s1);
        l_sum = l_sum * alpha + (s0 + s1);
      }
      // Rescale O when the max grew past the threshold (rare after the first tiles); PV_x(j)
      // cannot start before this group's P_x(j) arrival below, and PV_x(j-1) must have landed.
      if (__any_sync(0xffffffffu, alpha != 1.f)) {
        if (!__all_sync(0xffffffffu, wait_bar(&bars[kBarPVDone + x], (j - 1) & 1, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float v[32];
          tmem_ld32(tO[x] + lane_off + c * 32, v);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] *= alpha;
          tmem_st32(tO[x] + lane_off + c * 32, v);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars[kBarPFull + x]);
    }
    if (ok && nx > 0 &&
        __all_sync(0xffffffffu, wait_bar(&bars[kBarPVDone + x], (nx - 1) & 1, abort_flag))) {
      tc_fence_after();
      const float inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
      const bool write = qi < p.q_len;
      bf16* orow = p.out + static_cast<int64_t>(qi) * p.o_st + static_cast<int64_t>(head) * p.o_sh;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32(tO[x] + lane_off + c * 32, v);
        tmem_wait_ld();
        if (write) {
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8) {
            uint4 o4;
            o4.x = pack_bf16x2(v[q8 * 8 + 0] * inv, v[q8 * 8 + 1] * inv);
            o4.y = pack_bf16x2(v[q8 * 8 + 2] * inv, v[q8 * 8 + 3] * inv);
            o4.z = pack_bf16x2(v[q8 * 8 + 4] * inv, v[q8 * 8 + 5] * inv);
            o4.w = pack_bf16x2(v[q8 * 8 + 6] * inv, v[q8 * 8 + 7] * inv);
            *reinterpret_cast<uint4*>(orow + c * 32 + q8 * 8) = o4;
          }
        }
      }
    }
  }

  // ---- teardown ----
  tc_fence_before();
  __syncthreads();
  if (*abort_flag && tid == 0) {
    const unsigned long long t0 = globaltimer_ns();
    auto drain = [&](uint64_t* bar, uint32_t parity) {
      while (!mbar_try_wait(smem_u32(bar), parity) && globaltimer_ns() - t0 < kWaitLimitNs) {
      }
    };
    drain(&bars[kBarQ], 0);
    for (int t = max(0, counts[0] - kStages); t < counts[0]; ++t)
      drain(&bars[kBarKFull + t % kStages], (t / kStages) & 1);
    for (int t = max(0, counts[1] - kStages); t < counts[1]; ++t)
      drain(&bars[kBarVFull + t % kStages], (t / kStages) & 1);
    for (int x = 0; x < 2; ++x) {
      if (counts[2 + x] > 0) drain(&bars[kBarSFull + x], (counts[2 + x] - 1) & 1);
      if (counts[4 + x] > 0) drain(&bars[kBarPVDone + x], (counts[4 + x] - 1) & 1);
    }
  }
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols));
  }
}

}  // namespace pp

int build_map(CUtensorMap* map, const void* base, int64_t stride_tok, int64_t stride_head,
              int tokens, int heads, int* tok_coord) {
  if (stride_tok <= 0 || stride_head <= 0) return SOLORT_ERR_INVALID_ARGUMENT;
  uint64_t dims[3], strides[2];
  uint32_t box[3];
  dims[0] = kHD;
  box[0] = 64;
  if (stride_head < stride_tok) {
    *tok_coord = 2;
    dims[1] = heads;
    dims[2] = tokens;
    strides[0] = stride_head * 2;
    strides[1] = stride_tok * 2;
    box[1] = 1;
    box[2] = 128;
  } else {
    *tok_coord = 1;
    dims[1] = tokens;
    dims[2] = heads;
    strides[0] = stride_tok * 2;
    strides[1] = stride_head * 2;
    box[1] = 128;
    box[2] = 1;
  }
  return encode_bf16_map(map, base, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace pre

int read_prefill_status(unsigned* flags) {
  unsigned v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_prefill_status, sizeof(v)) != cudaSuccess) return SOLORT_ERR_CUDA;
  if (v && cudaMemcpyToSymbol(g_prefill_status, &zero, sizeof(zero)) != cudaSuccess)
    return SOLORT_ERR_CUDA;
  *flags |= v;
  return SOLORT_OK;
}

}  // namespace solort

using namespace solort;
using namespace solort::pre;

extern "C" int solort_attn_prefill(const SolortPrefillArgs* a, void* stream_v) {
  if (!a || !a->q || !a->k || !a->v || !a->out) return SOLORT_ERR_INVALID_ARGUMENT;
  if (a->head_dim != kHD) return SOLORT_ERR_UNSUPPORTED;
  if (a->q_len <= 0 || a->kv_len <= 0 || a->num_qo_heads <= 0 || a->num_kv_heads <= 0 ||
      a->num_qo_heads % a->num_kv_heads != 0)
    return SOLORT_ERR_INVALID_ARGUMENT;
  if (a->causal && a->q_len > a->kv_len) return SOLORT_ERR_INVALID_ARGUMENT;
  if (!aligned(a->out, 16) || (a->out_stride_token & 7) || (a->out_stride_head & 7))
    return SOLORT_ERR_INVALID_ARGUMENT;
  DeviceInfo di;
  int rc = current_device_info(&di);
  if (rc != SOLORT_OK) return rc;
  if (di.max_smem_optin < kSmemBytes) return SOLORT_ERR_UNSUPPORTED;
  CUtensorMap tq, tk, tv;
  int q_tc = 1, kv_tc = 1, tmp = 1;
  rc = build_map(&tq, a->q, a->q_stride_token, a->q_stride_head, a->q_len, a->num_qo_heads, &q_tc);
  if (rc != SOLORT_OK) return rc;
  rc = build_map(&tk, a->k, a->kv_stride_token, a->kv_stride_head, a->kv_len, a->num_kv_heads,
                 &kv_tc);
  if (rc != SOLORT_OK) return rc;
  rc = build_map(&tv, a->v, a->kv_stride_token, a->kv_stride_head, a->kv_len, a->num_kv_heads, &tmp);
  if (rc != SOLORT_OK) return rc;
  Params prm{};
  prm.out = static_cast<bf16*>(a->out);
  prm.o_st = a->out_stride_token;
  prm.o_sh = a->out_stride_head;
  prm.q_len = a->q_len;
  prm.kv_len = a->kv_len;
  prm.nh = a->num_qo_heads;
  prm.group = a->num_qo_heads / a->num_kv_heads;
  prm.q_tiles = (a->q_len + kBM - 1) / kBM;
  prm.causal = a->causal ? 1 : 0;
  prm.q_tok_coord = q_tc;
  prm.kv_tok_coord = kv_tc;
  prm.scale_log2 = a->scale * 1.4426950408889634f;
  // Long prompts: two query tiles per CTA in ping-pong (enough CTAs remain to fill the GPU).
  // Shorter ones with more (query tile, head) items than SMs: one persistent CTA per SM walking
  // its share of the items. Otherwise one CTA per item.
  const bool ping_pong = prm.q_tiles >= kPingPongMinTiles;
  const int64_t work = static_cast<int64_t>(ping_pong ? (prm.q_tiles + 1) / 2 : prm.q_tiles) *
                       a->num_qo_heads;
  if (work > (1ll << 31) - 1) return SOLORT_ERR_UNSUPPORTED;
  const bool persistent = !ping_pong && di.sm_count > 0 && work > di.sm_count;
  const int64_t grid = persistent ? di.sm_count : work;
  if (ping_pong && di.max_smem_optin < pp::kSmemBytes) return SOLORT_ERR_UNSUPPORTED;
  if (persistent && di.max_smem_optin < items::kSmemBytes) return SOLORT_ERR_UNSUPPORTED;
  static std::atomic<unsigned> configured{0};  // one bit per device ordinal < 32
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return SOLORT_ERR_CUDA;
  if (dev >= 32 || !(configured.load(std::memory_order_acquire) & (1u << dev))) {
    if (cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kSmemBytes) != cudaSuccess ||
        cudaFuncSetAttribute(pp::prefill_pp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             pp::kSmemBytes) != cudaSuccess ||
        cudaFuncSetAttribute(items::prefill_items_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             items::kSmemBytes) != cudaSuccess)
      return SOLORT_ERR_CUDA;
    if (dev < 32) configured.fetch_or(1u << dev, std::memory_order_release);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = ping_pong ? pp::kSmemBytes : persistent ? items::kSmemBytes : kSmemBytes;
  cfg.stream = static_cast<cudaStream_t>(stream_v);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e =
      ping_pong    ? cudaLaunchKernelEx(&cfg, pp::prefill_pp_kernel, tq, tk, tv, prm)
      : persistent ? cudaLaunchKernelEx(&cfg, items::prefill_items_kernel, tq, tk, tv, prm)
                   : cudaLaunchKernelEx(&cfg, prefill_kernel, tq, tk, tv, prm);
  if (e != cudaSuccess) return SOLORT_ERR_CUDA;
  return launch_status();
}
