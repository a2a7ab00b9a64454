// Split-KV GQA decode / verify for sm_100a, static or paged KV, with the log-sum-exp merge.
// Two split kernels share the plan, the partial layout and the merge: decode_kernel (mma.sync,
// below) for short splits, where a call is latency-bound, and decode_tc_kernel (tcgen05 / TMEM,
// further down) for long splits of at most four query rows, where the tile stream dominates.
//
// decode_kernel: one CTA per (key split, KV head, sequence). Its KV rows stream through a 7-stage
// ring of 16 KB shared-memory stages (32 tokens of K and V, two 64-dim halves each) filled by TMA
// tile loads (128-byte swizzle, only the boxes that hold keys of this split): 112 KB, so a split
// of up to 224 keys is requested in full at once and a CTA never waits for its own refill. An
// mbarrier per stage counts the bytes in. Every query row that reads this KV head -- the `group`
// heads of the group times q_len tokens, up to 32 rows -- is packed into m16 tensor-core tiles, so
// each K/V byte is read from HBM once and from shared memory once for all of them: nothing is
// expanded with repeat_interleave. Warps 0-1 take the even stages and warps 2-3 the odd ones, each
// warp a 16-token half; the pair that empties a stage refills it. QK^T and PV run on mma.sync (bf16 in, fp32 accumulate) with an fp32 online softmax in the exp2
// domain whose row max is a quad shuffle. The warps combine through shared memory; with one split
// the CTA writes the final rows, otherwise an fp32 partial (O, LSE) per row.
//
// merge_kernel: one CTA per output row; its threads split the partials between eight warps and
// issue every load of the row at once, then combine the warps' (max, sum, O) in shared memory.
//
// Both kernels are launched as programmatic dependents (PDL): each lets the next launch begin
// at its start and waits for its predecessor's completion (griddepcontrol.wait) before its first
// global-memory access, so launch latency and set-up overlap the previous kernel's tail while all
// data dependencies keep plain stream order.
//
// Splits are sized so the decode grid is two CTAs per SM. Semantics follow the reference's decode
// (src/solort/model/cuda_graph_executor.py:168,180-184: keys 0..pos visible), verify (:250: query
// i at vpos0+i sees keys <= vpos0+i) and the paged addressing of src/solort/cache/kv_cache.py:
// 136-149 (slot = block_table[pos // P] * P + pos % P).
#include <atomic>
#include <math.h>
#include <string.h>

#include "common.cuh"
#include "host_util.h"
#include "tcgen05.cuh"

namespace solort {

__device__ unsigned g_decode_status;

namespace dec {

constexpr int kHD = 128;
constexpr int kTile = 32;                   // tokens per stage
constexpr int kBox = 32;                    // token rows per TMA box (static caches)
constexpr int kHalfBytes = kTile * 128;     // 32 tokens x 64 dims bf16: 4 KB
constexpr int kKVBytes = 2 * kHalfBytes;    // one of K or V for a stage: 8 KB
constexpr int kStageBytes = 2 * kKVBytes;   // K + V: 16 KB
constexpr int kMaxStages = 7;               // 112 KB: a 224-key split is requested at once
// Stages requested before the PDL wait when the prefix is stable; the rest go out right after it
// (the last one after the query rows). Five, not six: the sixth is warp pair 1's last tile, which
// it reaches last, and holding it back leaves 4.6 MB less queued in front of the previous call's
// merge and release. L = 8192, 36-layer graph: 10.16 -> 9.98 us per call (2-4 early: 10.6-10.9).
constexpr int kEarlyStages = 5;
// HOLD instances (splits of 5 to 7 tiles that fit the ring, stable prefix): only kHoldEarlyStages
// go out before the wait, and the other stable tiles with the last stage once the query rows are
// staged. L = 8192, 36-layer graph, per call: 9.90 -> 9.56 us (3 / 5 / 6 stages early: 9.93 /
// 9.82 / 10.17 against 9.63 for 4 in one A/B run). Kept a separate instance because
// the same code in the instance the runner's two-tile splits use (where it issues exactly the same
// tiles) cost that step ~1 us per decode call.
constexpr int kHoldEarlyStages = 4;
// Two CTAs per SM: 228 KB of shared memory per SM, less 1 KB the hardware keeps per CTA.
constexpr int kSmemPerCta = 115712;
// After the ring: full barriers, flags, the tile last issued into each stage, block-table slice.
constexpr int kHdrBytes = kMaxStages * 8 + 8 + kMaxStages * 4;
constexpr int kWarps = 4;  // consumer warps (two pairs)
// Single-tile query blocks (MT == 1) add a fifth warp that only issues the initial TMA fills, so
// no consumer warp is held up while the copy engine accepts them; MT == 2 needs every register of
// a 128-thread CTA, so there thread 0 issues them.
template <int MT>
struct Shape {
  static constexpr bool kProducerWarp = MT == 1;
  static constexpr int kThreads = kProducerWarp ? 160 : 128;
};
constexpr int kMaxPagedChunk = 16384;       // tokens per split at most with a block table
constexpr int kMinSplitTiles = 2;           // default plans: at least 64 keys per split
constexpr int kSingleSplitKeys = 128;       // default plans: one split up to this many keys
constexpr int kMergeWarps = 8;
constexpr float kLn2 = 0.6931471805599453f;

struct Params {
  const bf16* q;
  int64_t q_sb, q_st, q_sh;
  // final output: bf16 rows, or fp32 rows + LSE when out_f32 != nullptr
  bf16* out;
  int64_t o_sb, o_st, o_sh;
  float* out_f32;
  float* lse_out;
  // split partials (num_splits > 1): [S][rows_total][hd] and [S][rows_total]
  float* part_o;
  float* part_lse;
  const int64_t* q_pos;
  const int32_t* q_lens;
  int64_t kv_pos_offset;
  const int32_t* block_table;
  int64_t bt_stride;
  int page_size, page_shift, box_rows, num_pages;
  int tok_coord;  // 1: map coords (d, tok, head, page); 2: (d, head, tok, page)
  int kv_limit;   // local keys that may be read at most
  int batch, q_len, nh, nkv, group;
  int chunk, num_splits;
  int q_vec16;  // q base and strides allow 16-byte loads
  int force_partial;  // one split still goes through the partials and the merge kernel
  int stages;  // ring depth: kMaxStages, or one less when a long block-table slice needs room
  int stable_prefix;  // q_pos, q_lens, block table and keys below q_pos precede the previous kernel
  float scale_log2;
};

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Write one 4-dim chunk of a finished row (row index R over all rows = (b, token, head)).
__device__ __forceinline__ void write_final(const Params& p, int R, int c, float4 v, float lse) {
  if (p.out_f32) {
    *reinterpret_cast<float4*>(p.out_f32 + static_cast<int64_t>(R) * kHD + c) = v;
    if (c == 0) p.lse_out[R] = lse;
  } else {
    const int h = R % p.nh, t = (R / p.nh) % p.q_len, b = R / (p.nh * p.q_len);
    bf16* o = p.out + b * p.o_sb + t * p.o_st + h * p.o_sh + c;
    uint2 pk;
    pk.x = pack_bf16x2(v.x, v.y);
    pk.y = pack_bf16x2(v.z, v.w);
    *reinterpret_cast<uint2*>(o) = pk;
  }
}

__device__ __forceinline__ void write_partial(const Params& p, int split, int rows_total, int R,
                                              int c, float4 v, float lse) {
  *reinterpret_cast<float4*>(p.part_o + (static_cast<int64_t>(split) * rows_total + R) * kHD + c) = v;
  if (c == 0) p.part_lse[static_cast<int64_t>(split) * rows_total + R] = lse;
}

template <int MT, bool PAGED, bool HOLD>
__global__ void __launch_bounds__(Shape<MT>::kThreads, 2)
    decode_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                  const Params p) {
  // The ring starts the dynamic shared memory, which must be 1024-aligned for the 128-byte
  // swizzle; the declaration asks for that and the kernel checks it (no spare room to re-align).
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* stages = smem_raw;
  const int nst = p.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + nst * kStageBytes);
  int* flags = reinterpret_cast<int*>(full + kMaxStages);  // [0] abort
  int* last_fill = flags + 2;                              // tile last issued into each stage
  int* bt_s = last_fill + kMaxStages;

  const int split = blockIdx.x;
  const int kvh = blockIdx.y;
  const int b = blockIdx.z;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int pair = warp >> 1;  // warps 0-1 take the even tiles, warps 2-3 the odd ones
  const int wip = warp & 1;    // 16-token half of the tile this warp takes
  // Stages are private to a pair: pair g owns stages g, g+2, g+4, ... (ns_pair of them) and its
  // j-th tile uses stage g + 2 (j % ns_pair). Each stage thus has one consumer, which waits for
  // its fills in the order they were issued, so a parity wait can never see a fill one phase
  // early. Tile t < nst lands in stage t.
  const int rows_total = p.batch * p.q_len * p.nh;
  const bool single = p.num_splits == 1 && !p.force_partial;
  constexpr int kThreads = Shape<MT>::kThreads;
  const bool consumer = warp < kWarps;
  const bool initial_issuer = Shape<MT>::kProducerWarp ? (warp == kWarps && lane == 0) : tid == 0;

  pdl_launch_dependents();
  if (smem_u32(smem_raw) & 1023u) {
    if (tid == 0) atomicOr(&g_decode_status, kDevErrSmemAlign);
    return;
  }
  if (tid == 0) {
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
    for (int s = 0; s < nst; ++s) {
      mbar_init(&full[s], 1);
      last_fill[s] = -1;
    }
    flags[0] = 0;
    fence_mbarrier_init();
  }
  // Inputs and the workspace may belong to the kernel before this one. With stable_prefix the
  // positions, the block table and the keys below q_pos were written before it, so they are read
  // (and those keys requested) before waiting; everything else waits as usual.
  const bool early = p.stable_prefix != 0;
  // Warm L2 with this CTA's query rows before waiting: only a cache hint (the rows themselves are
  // read after the wait, so a predecessor that writes them is still respected).
  if (consumer) {
    const int rows_alloc = p.q_len * p.group;
    for (int idx = tid; idx < rows_alloc * 2; idx += kWarps * 32) {
      const int r = idx >> 1;
      const bf16* src = p.q + b * p.q_sb + (r / p.group) * p.q_st +
                        (kvh * p.group + r % p.group) * p.q_sh + (idx & 1) * 64;
      asm volatile("prefetch.global.L2 [%0];" ::"l"(src));
    }
  }
  if (!early) pdl_wait();

  const long long qpos = p.q_pos[b];
  const int qlen_b = p.q_lens ? min(p.q_lens[b], p.q_len) : p.q_len;
  const int rows_b = qlen_b * p.group;
  long long kv_end_ll = qpos + qlen_b - p.kv_pos_offset;
  kv_end_ll = kv_end_ll < 0 ? 0 : kv_end_ll;
  kv_end_ll = kv_end_ll > p.kv_limit ? p.kv_limit : kv_end_ll;
  const int kv_end = static_cast<int>(kv_end_ll);
  const int t_begin = split * p.chunk;
  const int t_end = min(t_begin + p.chunk, kv_end);
  const int ntiles = t_end > t_begin ? (t_end - t_begin + kTile - 1) / kTile : 0;

  // Row index over all rows of query row r (token r / group, head kvh*group + r % group).
  auto out_row = [&](int r) {
    return (b * p.q_len + r / p.group) * p.nh + kvh * p.group + r % p.group;
  };

  if (ntiles == 0) {
    // Nothing visible in this split: an empty partial (O = 0, LSE = -inf), or zero final rows.
    if (early) pdl_wait();
    for (int idx = tid; idx < rows_b * (kHD / 4); idx += kThreads) {
      const int r = idx / (kHD / 4), c = (idx % (kHD / 4)) * 4;
      const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
      if (single)
        write_final(p, out_row(r), c, z, -INFINITY);
      else
        write_partial(p, split, rows_total, out_row(r), c, z, -INFINITY);
    }
    return;
  }

  int lp0 = 0;
  if (PAGED) {
    lp0 = t_begin >> p.page_shift;
    const int lp1 = (t_end - 1) >> p.page_shift;
    for (int i = tid; i <= lp1 - lp0; i += kThreads)
      bt_s[i] = p.block_table[b * p.bt_stride + lp0 + i];
  }
  __syncthreads();

  // Fill stage s with the boxes of tile `it` that hold keys of this split. Rows of the stage past
  // the split end keep stale contents; they are masked (K) or zeroed (V) below.
  auto issue = [&](int it, int s) {
    uint8_t* Ks = stages + s * kStageBytes;
    uint8_t* Vs = Ks + kKVBytes;
    const int t0 = t_begin + it * kTile;
    const int br = p.box_rows;
    const int nbox = min(kTile, t_end - t0 + br - 1) / br;  // boxes with at least one key
    last_fill[s] = it;
    mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(nbox * br * 128 * 4));
    for (int j = 0; j < nbox; ++j) {
      const int tok = t0 + j * br;
      int c1, c2, c3;
      if (!PAGED) {
        c1 = p.tok_coord == 1 ? tok : kvh;
        c2 = p.tok_coord == 1 ? kvh : tok;
        c3 = 0;
      } else {
        const int row = tok & (p.page_size - 1);
        c1 = p.tok_coord == 1 ? row : kvh;
        c2 = p.tok_coord == 1 ? kvh : row;
        c3 = bt_s[(tok >> p.page_shift) - lp0];
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        tma_load_4d(Ks + h * kHalfBytes + j * br * 128, &tmK, &full[s], h * 64, c1, c2, c3);
        tma_load_4d(Vs + h * kHalfBytes + j * br * 128, &tmV, &full[s], h * 64, c1, c2, c3);
      }
    }
  };

  // Every stage but the last is filled at once; the last one first carries this CTA's query rows.
  // Tiles whose keys all lie below q_pos go out before the wait when the prefix is stable.
  int defer_i = 0, defer_n = 0;  // HOLD: stable tiles held back until the query rows are staged
  if (initial_issuer) {
    const int n0 = ntiles < nst - 1 ? ntiles : nst - 1;
    int i = 0;
    if (early) {
      const long long stable_end = qpos - p.kv_pos_offset;  // local keys below it are stable
      const int n_early = HOLD ? kHoldEarlyStages : kEarlyStages;
      while (i < n0 && i < n_early && min(t_begin + (i + 1) * kTile, t_end) <= stable_end) {
        issue(i, i);
        ++i;
      }
      if (HOLD) {
        defer_i = i;
        while (i < n0 && min(t_begin + (i + 1) * kTile, t_end) <= stable_end) ++i;
        defer_n = i;
      }
    }
    if (early) pdl_wait();
    for (; i < n0; ++i) issue(i, i);  // HOLD: the tiles holding q_pos and later keys
  } else if (early) {
    pdl_wait();
  }

  // Query fragments (A operand, m16k16 per (mt, ks)). The 37-odd CTAs of a KV head all need the
  // same rows, so each CTA reads them once with coalesced 16-byte loads into the last stage
  // (128-byte XOR swizzle, 256 B per row) and builds the fragments with ldmatrix; scattered
  // per-lane loads of the same few L2 sectors from every CTA take microseconds. Every row of the
  // q_len tokens is loaded (valid memory); rows past this sequence's q_lens are masked below.
  uint32_t qa[MT][8][4];
  uint8_t* q_stage = stages + (nst - 1) * kStageBytes;
  if (consumer) {
    const int rows_alloc = p.q_len * p.group;
    for (int idx = tid; idx < MT * 16 * 16; idx += kWarps * 32) {
      const int r = idx >> 4, c = idx & 15;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (r < rows_alloc) {
        const int qi = r / p.group, h = kvh * p.group + r % p.group;
        const bf16* src = p.q + b * p.q_sb + qi * p.q_st + h * p.q_sh + c * 8;
        if (p.q_vec16) {
          v = *reinterpret_cast<const uint4*>(src);
        } else {
          const uint32_t* s32 = reinterpret_cast<const uint32_t*>(src);
          v = make_uint4(s32[0], s32[1], s32[2], s32[3]);
        }
      }
      *reinterpret_cast<uint4*>(q_stage + r * 256 + ((c >> 3) << 7) + (((c & 7) ^ (r & 7)) << 4)) = v;
    }
    fence_proxy_async_shared();  // these writes precede the stage's TMA fill
    asm volatile("bar.sync 3, %0;" ::"n"(kWarps * 32) : "memory");
    const uint32_t qs = smem_u32(q_stage);
    const int m = lane >> 3;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int row = mt * 16 + (lane & 7) + (m & 1) * 8;
        const int kc = 2 * ks + (m >> 1);
        ldmatrix_x4(qa[mt][ks][0], qa[mt][ks][1], qa[mt][ks][2], qa[mt][ks][3],
                    qs + row * 256 + ((kc >> 3) << 7) + (((kc & 7) ^ (row & 7)) << 4));
      }
    if (Shape<MT>::kProducerWarp)
      asm volatile("bar.arrive 4, %0;" ::"n"((kWarps + 1) * 32) : "memory");
    else
      asm volatile("bar.sync 4, %0;" ::"n"(kWarps * 32) : "memory");
  } else {
    __syncwarp();
    asm volatile("bar.sync 4, %0;" ::"n"((kWarps + 1) * 32) : "memory");
  }
  if (HOLD) {
    // The held-back tiles and the last stage from one issue site (each inlined copy of `issue` is a
    // few hundred bytes of the kernel's code).
    if (initial_issuer) {
      const int last = ntiles >= nst ? nst - 1 : -1;
      for (int t = defer_i; t < nst; ++t)
        if (t < defer_n || t == last) issue(t, t);
    }
  } else if (initial_issuer && ntiles >= nst) {
    issue(nst - 1, nst - 1);
  }

  int lim[MT][2];  // last visible local key of the two rows this lane holds per m-tile
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int r = mt * 16 + (lane >> 2) + hr * 8;
      if (r < rows_b) {
        long long last = qpos + r / p.group - p.kv_pos_offset;
        last = last < t_end - 1 ? last : t_end - 1;
        lim[mt][hr] = static_cast<int>(last < -1 ? -1 : last);
      } else {
        lim[mt][hr] = -1;
      }
    }
  }

  float m_run[MT][2], l_run[MT][2];
  float o_acc[MT][16][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      m_run[mt][hr] = -INFINITY;
      l_run[mt][hr] = 0.f;
    }
#pragma unroll
    for (int n = 0; n < 16; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) o_acc[mt][n][e] = 0.f;
  }

  // Two independent QK accumulator chains shorten the dependent mma sequence when registers allow.
  constexpr int kChains = MT == 1 ? 2 : 1;
  const uint32_t stages_u32 = smem_u32(stages);
  bool ok = true;
  const int ns_pair = (nst + 1 - pair) >> 1;
  for (int it = consumer ? pair : ntiles, j = 0; it < ntiles; it += 2, ++j) {
    const int s = pair + 2 * (j % ns_pair);
    const uint32_t parity = (j / ns_pair) & 1;
    if (!mbar_wait(&full[s], parity, &g_decode_status)) ok = false;
    ok = __all_sync(0xffffffffu, ok);  // the mma below needs every lane
    if (!ok) flags[0] = 1;
    const int tok0 = t_begin + it * kTile + wip * 16;
    if (ok && tok0 < t_end) {
      const uint32_t Ks = stages_u32 + s * kStageBytes;
      const uint32_t Vs = Ks + kKVBytes;
      if (t_end - tok0 < 16) {
        // Rows past the last key hold stale or never-written shared memory; their P is exactly
        // 0, but 0 * NaN is not, so zero this warp's V rows past the end.
        uint8_t* Vg = stages + s * kStageBytes + kKVBytes;
        const int valid = t_end - tok0;
        for (int idx = lane; idx < (16 - valid) * 16; idx += 32) {
          const int trow = wip * 16 + valid + (idx >> 4);
          const int ch = idx & 15;
          *reinterpret_cast<uint4*>(Vg + (ch >> 3) * kHalfBytes + swz128(trow, ch & 7)) =
              make_uint4(0u, 0u, 0u, 0u);
        }
        fence_proxy_async_shared();  // order these writes before the stage's next TMA fill
        __syncwarp();
      }
      float sc[kChains][MT][2][4];
#pragma unroll
      for (int ch = 0; ch < kChains; ++ch)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) sc[ch][mt][nt][e] = 0.f;
      // S = Q K^T over 128 dims: 8 k-steps, two n8 tiles of tokens.
      {
        const int mi = lane >> 3;
        const int trow = wip * 16 + ((mi >> 1) << 3) + (lane & 7);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const int half = ks >> 2;
          const int chunk = ((ks & 3) << 1) + (mi & 1);
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(b0, b1, b2, b3, Ks + half * kHalfBytes + swz128(trow, chunk));
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            mma_bf16_16816(sc[ks % kChains][mt][0], qa[mt][ks], b0, b1);
            mma_bf16_16816(sc[ks % kChains][mt][1], qa[mt][ks], b2, b3);
          }
        }
      }
#pragma unroll
      for (int ch = 1; ch < kChains; ++ch)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) sc[0][mt][nt][e] += sc[ch][mt][nt][e];
      // Mask, scale to the exp2 domain, online softmax.
      uint32_t pa[MT][4];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          float mx = -INFINITY;
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              const int tok = tok0 + nt * 8 + (lane & 3) * 2 + c;
              float v = sc[0][mt][nt][hr * 2 + c] * p.scale_log2;
              v = tok <= lim[mt][hr] ? v : -INFINITY;
              sc[0][mt][nt][hr * 2 + c] = v;
              mx = fmaxf(mx, v);
            }
          mx = warp_max_quad(mx);
          const float m_new = fmaxf(m_run[mt][hr], mx);
          const float ref = m_new == -INFINITY ? 0.f : m_new;
          const float alpha = exp2f(m_run[mt][hr] - ref);
          float rs = 0.f;
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              const float e = exp2f(sc[0][mt][nt][hr * 2 + c] - ref);
              sc[0][mt][nt][hr * 2 + c] = e;
              rs += e;
            }
          l_run[mt][hr] = l_run[mt][hr] * alpha + rs;
          m_run[mt][hr] = m_new;
#pragma unroll
          for (int n = 0; n < 16; ++n) {
            o_acc[mt][n][hr * 2] *= alpha;
            o_acc[mt][n][hr * 2 + 1] *= alpha;
          }
        }
        pa[mt][0] = pack_bf16x2(sc[0][mt][0][0], sc[0][mt][0][1]);
        pa[mt][1] = pack_bf16x2(sc[0][mt][0][2], sc[0][mt][0][3]);
        pa[mt][2] = pack_bf16x2(sc[0][mt][1][0], sc[0][mt][1][1]);
        pa[mt][3] = pack_bf16x2(sc[0][mt][1][2], sc[0][mt][1][3]);
      }
      // O += P V: V^T fragments via ldmatrix.trans, 16 n8 tiles of dims.
      {
        const int mi = lane >> 3;
        const int trow = wip * 16 + ((mi & 1) << 3) + (lane & 7);
#pragma unroll
        for (int dn = 0; dn < 8; ++dn) {
          const int dchunk = dn * 2 + (mi >> 1);
          uint32_t v0, v1, v2, v3;
          ldmatrix_x4_trans(v0, v1, v2, v3,
                            Vs + (dchunk >> 3) * kHalfBytes + swz128(trow, dchunk & 7));
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            mma_bf16_16816(o_acc[mt][2 * dn], pa[mt], v0, v1);
            mma_bf16_16816(o_acc[mt][2 * dn + 1], pa[mt], v2, v3);
          }
        }
      }
    }
    // Both warps of the pair are done with stage s: refill it with the pair's tile ns_pair on.
    // Without a refill (a split that fits the ring) the pair need not meet; the condition is the
    // same for both warps of the pair. An abort is seen by the pair at its next meeting or after
    // the loop.
    if (it + 2 * ns_pair < ntiles) {
      if (pair == 0)
        asm volatile("bar.sync 1, 64;" ::: "memory");
      else
        asm volatile("bar.sync 2, 64;" ::: "memory");
      if (flags[0]) break;
      if (wip == 0 && lane == 0) issue(it + 2 * ns_pair, s);
    } else if (flags[0]) {
      break;
    }
  }
  __syncthreads();

  if (flags[0]) {
    // A stage never completed within the time limit. The last fill of every stage may still have
    // copies in flight: give each a bounded wait before the CTA releases its shared memory, and
    // write nothing (the status word tells the host).
    if (tid == 0) {
      for (int st = 0; st < nst; ++st) {
        const int t = last_fill[st];
        if (t < 0) continue;
        const uint32_t bar = smem_u32(&full[st]);
        const uint32_t par = (((t >> 1) / ((nst + 1 - (t & 1)) >> 1))) & 1;
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(bar, par) && globaltimer_ns() - t0 < kWaitLimitNs) {
        }
      }
    }
    __syncthreads();
    return;
  }

  // ---- combine the four warps' (m, l, O) through shared memory ----
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) l_run[mt][hr] = warp_sum_quad(l_run[mt][hr]);

  // Latency matters here, not throughput (one short pass per CTA): each warp folds the
  // cross-warp max and the normaliser into one scale per row before it stores, so the last pass
  // only adds four vectors.
  constexpr int kRows = MT * 16;
  constexpr int kRedStride = kHD + 8;  // padded rows: each half-warp's float2 stores hit 32 banks
  float* red = reinterpret_cast<float*>(stages);  // [warps][kRows][kRedStride]
  float* ms = red + kWarps * kRows * kRedStride;   // [warps][kRows]
  float* ls = ms + kWarps * kRows;                 // [warps][kRows]
  float* lse_s = ls + kWarps * kRows;              // [kRows]
  if (consumer && (lane & 3) == 0) {
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const int r = mt * 16 + (lane >> 2) + hr * 8;
        if (r < rows_b) {
          ms[warp * kRows + r] = m_run[mt][hr];
          ls[warp * kRows + r] = l_run[mt][hr];
        }
      }
  }
  __syncthreads();
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int r = mt * 16 + (lane >> 2) + hr * 8;
      if (!consumer || r >= rows_b) continue;  // only live rows are combined
      float mw[kWarps];
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        mw[w] = ms[w * kRows + r];
        M = fmaxf(M, mw[w]);
      }
      float L = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w)
        L += mw[w] == -INFINITY ? 0.f : ls[w * kRows + r] * exp2f(mw[w] - M);
      // This warp's share of the normalised row: exp2(m_w - M) / L.
      const float f = (m_run[mt][hr] == -INFINITY || !(L > 0.f))
                          ? 0.f
                          : exp2f(m_run[mt][hr] - M) * __frcp_rn(L);
      if (warp == 0 && (lane & 3) == 0) lse_s[r] = L > 0.f ? (M + __log2f(L)) * kLn2 : -INFINITY;
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        const int c = n * 8 + (lane & 3) * 2;
        *reinterpret_cast<float2*>(red + (warp * kRows + r) * kRedStride + c) =
            make_float2(o_acc[mt][n][hr * 2] * f, o_acc[mt][n][hr * 2 + 1] * f);
      }
    }
  __syncthreads();

  for (int idx = tid; idx < rows_b * (kHD / 4); idx += kThreads) {
    const int r = idx / (kHD / 4), c = (idx % (kHD / 4)) * 4;
    float4 o = *reinterpret_cast<const float4*>(red + r * kRedStride + c);
#pragma unroll
    for (int w = 1; w < kWarps; ++w) {
      const float4 v = *reinterpret_cast<const float4*>(red + (w * kRows + r) * kRedStride + c);
      o.x += v.x;
      o.y += v.y;
      o.z += v.z;
      o.w += v.w;
    }
    if (single)
      write_final(p, out_row(r), c, o, lse_s[r]);
    else
      write_partial(p, split, rows_total, out_row(r), c, o, lse_s[r]);
  }
}

// ------------------------------------------------------------------------------------------
// decode_tc_kernel: the same split-KV decode on the 5th-generation tensor cores. The plan picks it
// for splits of at least kMinChunk keys with at most four query rows per KV head (RB, the
// compile-time row bound, is 4); there it streams a split's tiles faster than decode_kernel
// (131072 keys: 86.6 vs 89 us per layer). On short splits it loses: each 64-key tile costs ~1800
// cycles of hand-offs (QK commit -> TMEM load -> cross-warp row max -> P store -> PV issue),
// against decode_kernel's per-warp tile loop that needs no exchange until the end.
//
// The query rows are the narrow side, so both products are transposed: S^T = K Q^T with the keys
// as M (tcgen05.mma M = 64, N = 16 query rows, K = 128 dims) and O^T = V^T P^T with the head dims
// as M (M = 128, N = 16, K = 64 keys, V^T read as an MN-major operand straight from the TMA
// tiles). The tensor core reads K and V from shared memory itself -- no ldmatrix pass through the
// register file -- and its throughput makes the rows padded up to 16 cost little. S^T of a 64-key
// tile lands in TMEM with key m in lane (m % 16) + 32 (m / 16) (the M = 64 layout): warp w's
// lanes 0-15 hold keys 16w..16w+15, one column per query row. Four softmax warps read it, take
// the tile's row maxima (16-lane shuffles, then the four warps through shared memory), keep one
// running maximum per row with lazy rescaling (O in TMEM is rescaled only when a row's maximum
// grows by more than 2^64), and write P^T as bf16 for the PV MMA. One thread issues the MMAs, one
// the TMA copies. 64-key tiles cycle through a 3-tile ring (three 8 KB slots in each of four 24 KB
// regions: K dims 0-63, K dims 64-127, V dims 0-63, V dims 64-127); tiles past the ring are
// prefetched into L2 so their refill is an L2 read. At the end each thread owns one head dim of
// every row (O^T lane = dim), so the epilogue is one TMEM load, the row sums, and coalesced
// stores of the partial (O, LSE) or the final bf16 rows.
// ------------------------------------------------------------------------------------------
namespace tc {
constexpr int kTileKeys = 64;
constexpr int kSlots = 3;
constexpr int kRegionRows = kTileKeys * kSlots;  // 192
constexpr int kRegionBytes = kRegionRows * 128;  // 24 KB
constexpr int kSlotBytes = kTileKeys * 128;      // 8 KB
constexpr int kN = 16;                           // query rows per MMA
constexpr int kOffK0 = 0;
constexpr int kOffK1 = kRegionBytes;
constexpr int kOffV0 = 2 * kRegionBytes;
constexpr int kOffV1 = 3 * kRegionBytes;
constexpr int kQHalf = kN * 128;                  // one 64-dim half of the query rows: 2 KB
constexpr int kOffQ = 4 * kRegionBytes;           // 96 KB
constexpr int kPBytes = kN * 128;                 // P^T of one tile: 2 KB
constexpr int kOffP = kOffQ + 2 * kQHalf;         // two P buffers
constexpr int kOffHdr = kOffP + 2 * kPBytes;      // 104 KB
enum {
  kBarFull = 0,                        // +slot: TMA bytes of a tile landed
  kBarSFull = kBarFull + kSlots,       // +S buffer: QK committed
  kBarSFree = kBarSFull + 2,           // +S buffer: 128 softmax threads read it
  kBarPFull = kBarSFree + 2,           // +P buffer: 128 threads wrote P (and rescaled O)
  kBarPFree = kBarPFull + 2,           // +P buffer: PV committed
  kBarSlotFree = kBarPFree + 2,        // +slot: PV of the slot's tile committed
  kBarXMax = kBarSlotFree + kSlots,    // +tile parity: row maxima exchanged (128 arrivals)
  kBarXSum = kBarXMax + 2,             // row sums exchanged (128 arrivals)
  kBarQ = kBarXSum + 1,                // query rows staged (128 arrivals)
  kBarOFinal = kBarQ + 1,              // every MMA done
  kNumBars = kBarOFinal + 1
};
constexpr int kHdrInts = 8;  // [0] abort, [1] TMEM base, [2..4] tile last issued per slot
constexpr int kOffRedMax = kOffHdr + kNumBars * 8 + kHdrInts * 4;  // [2][4][kN] fp32
constexpr int kOffRedL = kOffRedMax + 2 * 4 * kN * 4;              // [4][kN] fp32
constexpr int kOffBt = kOffRedL + 4 * kN * 4;                      // block-table slice
constexpr int kThreads = 192;  // warps 0-3 softmax + epilogue, 4 MMA issue, 5 TMA producer
constexpr int kSoftmaxThreads = 128;
constexpr uint32_t kTmemCols = 64;  // S^T x 2 (16 columns each), O^T (16)
// Lazy rescaling: O^T in TMEM is rescaled only when a row's tile maximum exceeds the reference
// it was accumulated against by more than 2^64 (log2 domain). P <= 2^64 stays finite in bf16, and
// O and the row sums stay below 2^64 * (keys in the split) * max|v| in fp32, far inside its 2^128
// range for any split the plan makes (at most 2^31 keys) and |v| < 2^32; scores of a real
// model rarely move the maximum that much, so the pipeline-draining rescale almost never runs.
constexpr float kRescaleLog2 = 64.f;
constexpr int kMinChunk = 2048;  // keys per split from which the plan picks this kernel
constexpr uint32_t kIdescQK = umma::idesc_bf16(64, kN, false, false);
constexpr uint32_t kIdescPV = umma::idesc_bf16(128, kN, true, false);
static_assert(kOffBt % 4 == 0, "block-table slice alignment");
}  // namespace tc

// Bounded mbarrier wait that also gives up once another role has aborted.
// Waiting threads suspend in hardware (up to 20 us per try, resuming when the phase completes), so
// the MMA-issue and TMA threads do not take issue slots from the softmax warps while they wait.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait_suspend(addr, parity, 20000u)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      atomicOr(&g_decode_status, kDevErrBarrierTimeout);
      *abort_flag = 1;
      return false;
    }
  }
}

// One element of a finished row: bf16 output, or fp32 output + LSE (partial-output mode).
__device__ __forceinline__ void write_final1(const Params& p, int R, int d, float v, float lse) {
  if (p.out_f32) {
    p.out_f32[static_cast<int64_t>(R) * kHD + d] = v;
    if (d == 0) p.lse_out[R] = lse;
  } else {
    const int h = R % p.nh, t = (R / p.nh) % p.q_len, b = R / (p.nh * p.q_len);
    p.out[b * p.o_sb + t * p.o_st + h * p.o_sh + d] = __float2bfloat16_rn(v);
  }
}

template <bool PAGED, int RB>
__global__ void __launch_bounds__(tc::kThreads, 2)
    decode_tc_kernel(const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const Params p) {
  using namespace tc;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = smem_raw;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kOffHdr);
  int* hdr = reinterpret_cast<int*>(bars + kNumBars);
  volatile int* abort_flag = hdr;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(hdr + 1);
  int* last_fill = hdr + 2;
  float* red_max = reinterpret_cast<float*>(sm + kOffRedMax);
  float* red_l = reinterpret_cast<float*>(sm + kOffRedL);
  int* bt_s = reinterpret_cast<int*>(sm + kOffBt);
  const uint32_t sbase = smem_u32(sm);

  const int split = blockIdx.x;
  const int kvh = blockIdx.y;
  const int b = blockIdx.z;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int rows_total = p.batch * p.q_len * p.nh;
  const bool single = p.num_splits == 1 && !p.force_partial;

  if (sbase & 1023u) {
    if (tid == 0) atomicOr(&g_decode_status, kDevErrSmemAlign);
    return;
  }
  if (tid == 0) {
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
    for (int i = 0; i < kNumBars; ++i) {
      const bool many = (i >= kBarSFree && i < kBarSFree + 2) || (i >= kBarPFull && i < kBarPFull + 2) ||
                        (i >= kBarXMax && i < kBarXSum + 1) || i == kBarQ;
      mbar_init(&bars[i], many ? kSoftmaxThreads : 1);
    }
    hdr[0] = 0;
    for (int s = 0; s < kSlots; ++s) last_fill[s] = -1;
    fence_mbarrier_init();
  }
  const bool early = p.stable_prefix != 0;
  if (warp < 4) {  // warm L2 with the query rows (a hint: they are read after the wait)
    for (int idx = tid; idx < p.q_len * p.group * 2; idx += kSoftmaxThreads) {
      const int r = idx >> 1;
      const bf16* src = p.q + b * p.q_sb + (r / p.group) * p.q_st +
                        (kvh * p.group + r % p.group) * p.q_sh + (idx & 1) * 64;
      asm volatile("prefetch.global.L2 [%0];" ::"l"(src));
    }
  }
  if (!early) pdl_wait();

  const long long qpos = p.q_pos[b];
  const int qlen_b = p.q_lens ? min(p.q_lens[b], p.q_len) : p.q_len;
  const int rows_b = qlen_b * p.group;
  long long kv_end_ll = qpos + qlen_b - p.kv_pos_offset;
  kv_end_ll = kv_end_ll < 0 ? 0 : kv_end_ll;
  kv_end_ll = kv_end_ll > p.kv_limit ? p.kv_limit : kv_end_ll;
  const int kv_end = static_cast<int>(kv_end_ll);
  const int t_begin = split * p.chunk;
  const int t_end = min(t_begin + p.chunk, kv_end);
  const int ntiles = t_end > t_begin ? (t_end - t_begin + kTileKeys - 1) / kTileKeys : 0;
  auto out_row = [&](int r) {
    return (b * p.q_len + r / p.group) * p.nh + kvh * p.group + r % p.group;
  };

  if (ntiles == 0) {
    // Nothing visible in this split: an empty partial (O = 0, LSE = -inf), or zero final rows.
    if (early) pdl_wait();
    for (int idx = tid; idx < rows_b * kHD; idx += kThreads) {
      const int r = idx / kHD, d = idx % kHD;
      if (single)
        write_final1(p, out_row(r), d, 0.f, -INFINITY);
      else {
        p.part_o[(static_cast<int64_t>(split) * rows_total + out_row(r)) * kHD + d] = 0.f;
        if (d == 0) p.part_lse[static_cast<int64_t>(split) * rows_total + out_row(r)] = -INFINITY;
      }
    }
    return;
  }

  int lp0 = 0;
  if (PAGED) {
    lp0 = t_begin >> p.page_shift;
    const int lp1 = (t_end - 1) >> p.page_shift;
    for (int i = tid; i <= lp1 - lp0; i += kThreads)
      bt_s[i] = p.block_table[b * p.bt_stride + lp0 + i];
  }
  if (warp == 0) umma::alloc(tmem_slot, kTmemCols);
  umma::fence_before();
  __syncthreads();
  umma::fence_after();
  // The next kernel may launch once every CTA holds its TMEM (a dependent CTA that took the
  // columns first would wait on this grid while this CTA waited on the columns).
  pdl_launch_dependents();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tO = tmem + 2 * kN;

  // TMA coordinates of the box of `tok` rows (map coordinate order as the tensor maps define).
  auto coords = [&](int tok, int& c1, int& c2, int& c3) {
    if (!PAGED) {
      c1 = p.tok_coord == 1 ? tok : kvh;
      c2 = p.tok_coord == 1 ? kvh : tok;
      c3 = 0;
    } else {
      const int row = tok & (p.page_size - 1);
      c1 = p.tok_coord == 1 ? row : kvh;
      c2 = p.tok_coord == 1 ? kvh : row;
      c3 = bt_s[(tok >> p.page_shift) - lp0];
    }
  };
  // Fill slot s with the boxes of tile `it` that hold keys of this split; rows of the slot past
  // the split end keep stale contents (masked for K, zeroed for V before the PV MMA).
  auto issue = [&](int it, int s) {
    const int t0 = t_begin + it * kTileKeys;
    const int br = p.box_rows;
    const int nbox = (min(kTileKeys, t_end - t0) + br - 1) / br;
    last_fill[s] = it;
    mbar_arrive_expect_tx(&bars[kBarFull + s], static_cast<uint32_t>(nbox * br * 128 * 4));
    for (int j = 0; j < nbox; ++j) {
      int c1, c2, c3;
      coords(t0 + j * br, c1, c2, c3);
      const int off = s * kSlotBytes + j * br * 128;
      tma_load_4d(sm + kOffK0 + off, &tmK, &bars[kBarFull + s], 0, c1, c2, c3);
      tma_load_4d(sm + kOffK1 + off, &tmK, &bars[kBarFull + s], 64, c1, c2, c3);
      tma_load_4d(sm + kOffV0 + off, &tmV, &bars[kBarFull + s], 0, c1, c2, c3);
      tma_load_4d(sm + kOffV1 + off, &tmV, &bars[kBarFull + s], 64, c1, c2, c3);
    }
  };
  auto prefetch = [&](int it) {
    const int t0 = t_begin + it * kTileKeys;
    const int br = p.box_rows;
    const int nbox = (min(kTileKeys, t_end - t0) + br - 1) / br;
    for (int j = 0; j < nbox; ++j) {
      int c1, c2, c3;
      coords(t0 + j * br, c1, c2, c3);
      tma_prefetch_l2_4d(&tmK, 0, c1, c2, c3);
      tma_prefetch_l2_4d(&tmK, 64, c1, c2, c3);
      tma_prefetch_l2_4d(&tmV, 0, c1, c2, c3);
      tma_prefetch_l2_4d(&tmV, 64, c1, c2, c3);
    }
  };

  if (warp == 5) {
    // ---- TMA producer ----
    if (lane == 0) {
      const int n0 = min(ntiles, kSlots);
      const int pre_end = min(ntiles, 2 * kSlots);
      int i = 0;
      if (early) {
        // Tiles whose keys all lie below q_pos were written before the previous kernel.
        const long long stable_end = qpos - p.kv_pos_offset;
        while (i < n0 && min(t_begin + (i + 1) * kTileKeys, t_end) <= stable_end) {
          issue(i, i);
          ++i;
        }
        for (int it = kSlots; it < pre_end; ++it)
          if (min(t_begin + (it + 1) * kTileKeys, t_end) <= stable_end) prefetch(it);
        pdl_wait();
      }
      for (; i < n0; ++i) issue(i, i);
      if (!early)
        for (int it = kSlots; it < pre_end; ++it) prefetch(it);
      for (int t = kSlots; t < ntiles; ++t) {
        const int s = t % kSlots;
        if (!tc_wait(&bars[kBarSlotFree + s], ((t - kSlots) / kSlots) & 1, abort_flag)) break;
        issue(t, s);
        if (t + kSlots < ntiles) prefetch(t + kSlots);
      }
    }
    __syncwarp();
  } else if (warp == 4) {
    // ---- MMA issuer ----
    if (lane == 0) {
      bool ok = tc_wait(&bars[kBarQ], 0, abort_flag);
      auto pv = [&](int u) -> bool {
        const int bu = u & 1, su = u % kSlots;
        if (!tc_wait(&bars[kBarPFull + bu], (u >> 1) & 1, abort_flag)) return false;
        umma::fence_after();
#pragma unroll
        for (int kk = 0; kk < kTileKeys / 16; ++kk) {
          // V^T: MN-major (dims contiguous), 16 keys = two 8-row groups; the 64-dim halves are
          // one region apart. P^T: K-major, 16 keys = 32 bytes of each 128-byte row.
          const uint64_t da = umma::smem_desc(sbase + kOffV0 + su * kSlotBytes + kk * 2048,
                                              kRegionBytes, 1024);
          const uint64_t db = umma::smem_desc(sbase + kOffP + bu * kPBytes + kk * 32, 16, 1024);
          umma::mma_ss(tO, da, db, kIdescPV, (u > 0 || kk > 0) ? 1u : 0u);
        }
        umma::commit(&bars[kBarSlotFree + su]);
        umma::commit(&bars[kBarPFree + bu]);
        return true;
      };
      for (int t = 0; ok && t < ntiles; ++t) {
        const int s = t % kSlots, bb = t & 1;
        if (!tc_wait(&bars[kBarFull + s], (t / kSlots) & 1, abort_flag) ||
            (t >= 2 && !tc_wait(&bars[kBarSFree + bb], ((t - 2) >> 1) & 1, abort_flag))) {
          ok = false;
          break;
        }
        umma::fence_after();
#pragma unroll
        for (int kk = 0; kk < kHD / 16; ++kk) {
          const uint32_t ka = (kk < 4 ? kOffK0 : kOffK1) + s * kSlotBytes + (kk & 3) * 32;
          const uint32_t qb = kOffQ + (kk >> 2) * kQHalf + (kk & 3) * 32;
          umma::mma_ss(tmem + bb * kN, umma::smem_desc(sbase + ka, 16, 1024),
                       umma::smem_desc(sbase + qb, 16, 1024), kIdescQK, kk > 0 ? 1u : 0u);
        }
        umma::commit(&bars[kBarSFull + bb]);
        if (t >= 1 && !pv(t - 1)) ok = false;
      }
      if (ok) pv(ntiles - 1);
      umma::commit(&bars[kBarOFinal]);  // arrives once every MMA issued above has completed
    }
    __syncwarp();
  } else {
    // ---- softmax + epilogue (warps 0-3) ----
    // Every per-row sequence below is written step-major (all rows' shuffles of one step, all
    // loads before their uses) so that the rows' latency chains overlap; RB bounds the live rows
    // at compile time.
    if (early) pdl_wait();
    // Query rows into the B operand of S^T = K Q^T: K-major, 128-byte swizzle, two 64-dim halves;
    // rows past q_len * group are zero.
    const int rows_alloc = p.q_len * p.group;
    for (int idx = tid; idx < kN * 16; idx += kSoftmaxThreads) {
      const int r = idx >> 4, c = idx & 15;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (r < rows_alloc) {
        const bf16* src = p.q + b * p.q_sb + (r / p.group) * p.q_st +
                          (kvh * p.group + r % p.group) * p.q_sh + c * 8;
        if (p.q_vec16) {
          v = *reinterpret_cast<const uint4*>(src);
        } else {
          const uint32_t* s32 = reinterpret_cast<const uint32_t*>(src);
          v = make_uint4(s32[0], s32[1], s32[2], s32[3]);
        }
      }
      *reinterpret_cast<uint4*>(sm + kOffQ + (c >> 3) * kQHalf + (r >> 3) * 1024 + (r & 7) * 128 +
                                (((c & 7) ^ (r & 7)) << 4)) = v;
    }
    fence_proxy_async_shared();
    mbar_arrive(&bars[kBarQ]);

    int lim[RB];  // last visible local key of each row (-1: none)
    float m_run[RB], l_part[RB];
#pragma unroll
    for (int r = 0; r < RB; ++r) {
      long long last = qpos + r / p.group - p.kv_pos_offset;
      last = last < t_end - 1 ? last : t_end - 1;
      lim[r] = r < rows_b ? static_cast<int>(last < -1 ? -1 : last) : -1;
      m_run[r] = -INFINITY;
      l_part[r] = 0.f;
    }
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const int kl = warp * 16 + lane;  // this lane's key within a tile (lanes 0-15)
    bool ok = true;
    for (int t = 0; t < ntiles; ++t) {
      const int bb = t & 1, s = t % kSlots;
      if (!__all_sync(0xffffffffu, tc_wait(&bars[kBarSFull + bb], (t >> 1) & 1, abort_flag))) {
        ok = false;
        break;
      }
      umma::fence_after();
      float sv[16];
      if (RB <= 4)
        umma::ld4(tmem + bb * kN + lane_off, sv);
      else
        umma::ld16(tmem + bb * kN + lane_off, sv);
      umma::wait_ld();
      umma::fence_before();
      mbar_arrive(&bars[kBarSFree + bb]);
      const int key = t_begin + t * kTileKeys + kl;
      float v[RB], m[RB];
#pragma unroll
      for (int r = 0; r < RB; ++r) {
        v[r] = (lane < 16 && key <= lim[r]) ? sv[r] * p.scale_log2 : -INFINITY;
        m[r] = v[r];
      }
      // tile row maxima: 16 lanes, then the four warps through shared memory
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) {
        float x[RB];
#pragma unroll
        for (int r = 0; r < RB; ++r) x[r] = __shfl_xor_sync(0xffffffffu, m[r], o);
#pragma unroll
        for (int r = 0; r < RB; ++r) m[r] = fmaxf(m[r], x[r]);
      }
      float* rm = red_max + bb * 4 * kN;
      if (lane == 0) {
#pragma unroll
        for (int r = 0; r < RB; ++r) rm[warp * kN + r] = m[r];
      }
      mbar_arrive(&bars[kBarXMax + bb]);
      if (!__all_sync(0xffffffffu, tc_wait(&bars[kBarXMax + bb], (t >> 1) & 1, abort_flag))) {
        ok = false;
        break;
      }
      float w4[4][RB];
#pragma unroll
      for (int w = 0; w < 4; ++w)
#pragma unroll
        for (int r = 0; r < RB; ++r) w4[w][r] = rm[w * kN + r];
      bool grow = false;
      float alpha[RB];
#pragma unroll
      for (int r = 0; r < RB; ++r) {
        const float mt = fmaxf(fmaxf(w4[0][r], w4[1][r]), fmaxf(w4[2][r], w4[3][r]));
        const float mo = m_run[r];
        alpha[r] = 1.f;
        if (mt > -INFINITY && (mo == -INFINITY || mt > mo + kRescaleLog2)) {
          m_run[r] = mt;
          if (mo != -INFINITY) {
            alpha[r] = exp2f(mo - mt);
            grow = true;
          }
        }
      }
      if (grow) {
        // O^T holds the PV of tiles < t against the old maxima: wait for PV_{t-1}, rescale.
        if (!__all_sync(0xffffffffu, tc_wait(&bars[kBarSlotFree + (t - 1) % kSlots],
                                             ((t - 1) / kSlots) & 1, abort_flag))) {
          ok = false;
          break;
        }
        umma::fence_after();
        float ov[kN];
        umma::ld16(tO + lane_off, ov);
        umma::wait_ld();
#pragma unroll
        for (int r = 0; r < RB; ++r) ov[r] *= alpha[r];
        umma::st16(tO + lane_off, ov);
        umma::wait_st();
#pragma unroll
        for (int r = 0; r < RB; ++r) l_part[r] *= alpha[r];
      }
      float e[RB];
#pragma unroll
      for (int r = 0; r < RB; ++r) {
        e[r] = v[r] == -INFINITY ? 0.f : exp2f(v[r] - m_run[r]);
        l_part[r] += e[r];
      }
      // P buffer bb was last read by PV_{t-2}.
      if (t >= 2 && !__all_sync(0xffffffffu,
                                tc_wait(&bars[kBarPFree + bb], ((t - 2) >> 1) & 1, abort_flag))) {
        ok = false;
        break;
      }
      // P^T rows past RB feed O^T columns nobody reads and stay unwritten.
      uint8_t* pbuf = sm + kOffP + bb * kPBytes;
      if (lane < 16) {
#pragma unroll
        for (int r = 0; r < RB; ++r)
          *reinterpret_cast<bf16*>(pbuf + (r >> 3) * 1024 + (r & 7) * 128 +
                                   (((kl >> 3) ^ (r & 7)) << 4) + (kl & 7) * 2) =
              __float2bfloat16_rn(e[r]);
      }
      // Rows of the slot past the split end hold stale data: P is 0 there, but 0 * NaN is not,
      // so zero those V rows before the PV MMA reads them.
      const int valid = t_end - (t_begin + t * kTileKeys);
      if (valid < kTileKeys) {
        for (int idx = tid; idx < (kTileKeys - valid) * 16; idx += kSoftmaxThreads) {
          const int row = valid + (idx >> 4), c = idx & 15;
          uint8_t* vb = sm + ((c >> 3) ? kOffV1 : kOffV0) + s * kSlotBytes;
          *reinterpret_cast<uint4*>(vb + row * 128 + (((c & 7) ^ (row & 7)) << 4)) =
              make_uint4(0u, 0u, 0u, 0u);
        }
      }
      fence_proxy_async_shared();
      umma::fence_before();
      mbar_arrive(&bars[kBarPFull + bb]);
    }

    if (ok && !__all_sync(0xffffffffu, tc_wait(&bars[kBarOFinal], 0, abort_flag))) ok = false;
    if (ok) {
      umma::fence_after();
      float ov[16];
      if (RB <= 4)
        umma::ld4(tO + lane_off, ov);
      else
        umma::ld16(tO + lane_off, ov);
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) {
        float x[RB];
#pragma unroll
        for (int r = 0; r < RB; ++r) x[r] = __shfl_xor_sync(0xffffffffu, l_part[r], o);
#pragma unroll
        for (int r = 0; r < RB; ++r) l_part[r] += x[r];
      }
      if (lane == 0) {
#pragma unroll
        for (int r = 0; r < RB; ++r) red_l[warp * kN + r] = l_part[r];
      }
      umma::wait_ld();
      mbar_arrive(&bars[kBarXSum]);
      if (__all_sync(0xffffffffu, tc_wait(&bars[kBarXSum], 0, abort_flag))) {
        float w4[4][RB];
#pragma unroll
        for (int w = 0; w < 4; ++w)
#pragma unroll
          for (int r = 0; r < RB; ++r) w4[w][r] = red_l[w * kN + r];
        const int d = warp * 32 + lane;  // O^T lane = head dim
#pragma unroll
        for (int r = 0; r < RB; ++r) {
          if (r < rows_b) {
            const float L = (w4[0][r] + w4[1][r]) + (w4[2][r] + w4[3][r]);
            const float val = L > 0.f ? ov[r] * __frcp_rn(L) : 0.f;
            const float lse = L > 0.f ? (m_run[r] + __log2f(L)) * kLn2 : -INFINITY;
            const int R = out_row(r);
            if (single) {
              write_final1(p, R, d, val, lse);
            } else {
              p.part_o[(static_cast<int64_t>(split) * rows_total + R) * kHD + d] = val;
              if (d == 0) p.part_lse[static_cast<int64_t>(split) * rows_total + R] = lse;
            }
          }
        }
      }
    }
  }

  // ---- teardown: nothing may be in flight when the CTA releases TMEM and shared memory ----
  umma::fence_before();
  __syncthreads();
  if (*abort_flag && tid == 0) {
    const unsigned long long t0 = globaltimer_ns();
    auto drain = [&](uint64_t* bar, uint32_t parity) {
      while (!mbar_try_wait(smem_u32(bar), parity) && globaltimer_ns() - t0 < kWaitLimitNs) {
      }
    };
    for (int s = 0; s < kSlots; ++s)
      if (last_fill[s] >= 0) drain(&bars[kBarFull + s], (last_fill[s] / kSlots) & 1);
    drain(&bars[kBarOFinal], 0);
  }
  __syncthreads();
  umma::fence_after();
  if (warp == 0) umma::dealloc(tmem, kTmemCols);
}

struct MergeParams {
  const float* o_parts;
  int64_t part_stride;
  const float* lse_parts;
  int64_t lse_part_stride;
  int num_parts;
  int rows_total;
  const int32_t* q_lens;  // optional: rows whose token index is past q_lens[b] are skipped
  Params out;             // output fields only (out / out_f32 / lse_out, strides, q_len, nh)
  // Exchange mode (n_dest > 0): instead of `out`, each row goes to n_dest slots of tagged 64-bit
  // words [rows*128 O][rows LSE] (peer memory for all but this rank).
  int n_dest;
  unsigned long long* dest[SOLORT_MAX_RANKS];
};

// One exchange word: the arrival mark in the high half, the float's bits in the low half, written
// by a single 64-bit store (single-copy atomic), so a reader that sees the mark sees the value.
__device__ __forceinline__ void store_tagged(unsigned long long* w, float v) {
  const unsigned long long x = (1ull << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(w), "l"(x) : "memory");
}

// One CTA per output row, 8 warps; warp g takes parts g, g+8, ... and lane l dims 4l..4l+3.
// Every thread issues all of its loads before using any, so a row costs one round trip.
__global__ void __launch_bounds__(kMergeWarps * 32) merge_kernel(const MergeParams p) {
  __shared__ float sm_m[kMergeWarps], sm_d[kMergeWarps];
  __shared__ float4 sm_o[kMergeWarps][32];
  const int R = blockIdx.x;
  const int g = threadIdx.x >> 5, lane = threadIdx.x & 31, c = lane * 4;
  pdl_launch_dependents();
  pdl_wait();
  if (p.q_lens) {
    const int t = (R / p.out.nh) % p.out.q_len, b = R / (p.out.nh * p.out.q_len);
    if (t >= p.q_lens[b]) return;
  }
  float m = -INFINITY, den = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  constexpr int kBatch = 8;  // parts per warp loaded together
  for (int s0 = g; s0 < p.num_parts; s0 += kMergeWarps * kBatch) {
    float l[kBatch];
    float4 v[kBatch];
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      const int s = s0 + i * kMergeWarps;
      if (s < p.num_parts) {
        l[i] = __ldcg(p.lse_parts + s * p.lse_part_stride + R);
        v[i] = __ldcg(reinterpret_cast<const float4*>(p.o_parts + s * p.part_stride +
                                                      static_cast<int64_t>(R) * kHD + c));
      } else {
        l[i] = -INFINITY;
        v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    float mb = m;
#pragma unroll
    for (int i = 0; i < kBatch; ++i) mb = fmaxf(mb, l[i]);
    if (mb != -INFINITY) {
      const float a = __expf(m - mb);  // m == -inf gives 0: nothing accumulated yet
      den *= a;
      acc.x *= a;
      acc.y *= a;
      acc.z *= a;
      acc.w *= a;
#pragma unroll
      for (int i = 0; i < kBatch; ++i) {
        const float w = __expf(l[i] - mb);
        den += w;
        acc.x += w * v[i].x;
        acc.y += w * v[i].y;
        acc.z += w * v[i].z;
        acc.w += w * v[i].w;
      }
      m = mb;
    }
  }
  if (lane == 0) {
    sm_m[g] = m;
    sm_d[g] = den;
  }
  sm_o[g][lane] = acc;
  __syncthreads();
  if (g != 0) return;
  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < kMergeWarps; ++w) M = fmaxf(M, sm_m[w]);
  float D = 0.f;
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
  if (M != -INFINITY) {
#pragma unroll
    for (int w = 0; w < kMergeWarps; ++w) {
      if (sm_m[w] == -INFINITY) continue;
      const float f = __expf(sm_m[w] - M);
      const float4 x = sm_o[w][lane];
      D += sm_d[w] * f;
      o.x += x.x * f;
      o.y += x.y * f;
      o.z += x.z * f;
      o.w += x.w * f;
    }
  }
  const float inv = D > 0.f ? __frcp_rn(D) : 0.f;
  const float4 res = make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
  const float lse = D > 0.f ? M + __logf(D) : -INFINITY;
  if (p.n_dest == 0) {
    write_final(p.out, R, c, res, lse);
    return;
  }
  // Exchange: the row goes into every rank's slot as tagged words (NVLink stores for peers); the
  // marks make the words self-announcing, so no fence or flag follows.
  for (int d = 0; d < p.n_dest; ++d) {
    unsigned long long* w = p.dest[d] + static_cast<int64_t>(R) * kHD + c;
    store_tagged(w + 0, res.x);
    store_tagged(w + 1, res.y);
    store_tagged(w + 2, res.z);
    store_tagged(w + 3, res.w);
    if (lane == 0) store_tagged(p.dest[d] + static_cast<int64_t>(p.rows_total) * kHD + R, lse);
  }
}

// ------------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------------

struct Plan {
  int mt = 1;
  bool tc = false;  // up to 16 query rows per KV head: the tcgen05 kernel
  bool paged = false;
  int kv_limit = 0;
  int chunk = 0;
  int splits = 0;
  int stages = kMaxStages;
  bool force_partial = false;  // exchange calls always merge through the partials
  bool hold = false;           // decode_kernel holds stable tiles back (see kHoldEarlyStages)
  size_t part_o_bytes = 0;
  size_t part_lse_bytes = 0;
  size_t ws_bytes = 0;
  size_t smem_bytes = 0;
  int rows_total = 0;
};

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

int make_plan(const SolortDecodeArgs* a, Plan* pl, bool force_partial = false) {
  if (!a || !pl) return SOLORT_ERR_INVALID_ARGUMENT;
  if (a->head_dim != kHD) return SOLORT_ERR_UNSUPPORTED;
  if (a->batch <= 0 || a->q_len <= 0 || a->num_qo_heads <= 0 || a->num_kv_heads <= 0)
    return SOLORT_ERR_INVALID_ARGUMENT;
  if (a->num_qo_heads % a->num_kv_heads != 0) return SOLORT_ERR_INVALID_ARGUMENT;
  if (a->batch > 65535 || a->num_kv_heads > 65535) return SOLORT_ERR_UNSUPPORTED;
  const int group = a->num_qo_heads / a->num_kv_heads;
  const int rows = a->q_len * group;
  if (rows > 32) return SOLORT_ERR_UNSUPPORTED;
  pl->mt = rows <= 16 ? 1 : 2;
  pl->tc = false;  // decided below, once the split length is known
  pl->paged = a->block_table != nullptr;
  if (a->max_kv_len <= 0) return SOLORT_ERR_INVALID_ARGUMENT;
  if (pl->paged) {
    const int P = a->page_size;
    if (P < 8 || (P & (P - 1)) != 0) return SOLORT_ERR_INVALID_ARGUMENT;
    if (a->num_pages <= 0) return SOLORT_ERR_INVALID_ARGUMENT;
    pl->kv_limit = a->max_kv_len;
  } else {
    if (a->kv_capacity <= 0) return SOLORT_ERR_INVALID_ARGUMENT;
    pl->kv_limit = a->max_kv_len < a->kv_capacity ? a->max_kv_len : a->kv_capacity;
  }
  DeviceInfo di;
  int rc = current_device_info(&di);
  if (rc != SOLORT_OK) return rc;
  // Two CTAs per SM are resident; size the splits so the grid is one such wave.
  const int64_t resident = 2ll * di.sm_count;
  const int64_t heads = static_cast<int64_t>(a->batch) * a->num_kv_heads;
  // One resident wave of splits, but at least kMinSplitTiles tiles per split (a one-tile split is
  // all fixed cost and one more partial for the merge), and a single split, with no merge, up to
  // kSingleSplitKeys keys. Measured per call (32/8 heads, stable prefix): 64-key splits against
  // 128-key ones take L = 1024 from 6.76 to 5.98 us and L = 512 from 6.20 to 5.98; at L = 128 two
  // splits and a merge take 5.2 us against 3.6 for one split.
  const int64_t wave = resident / heads > 1 ? resident / heads : 1;
  const int64_t by_len = pl->kv_limit <= kSingleSplitKeys
                             ? 1
                             : ceil_div(pl->kv_limit, static_cast<int64_t>(kMinSplitTiles) * kTile);
  const int64_t target = a->num_splits > 0 ? a->num_splits : (by_len < wave ? by_len : wave);
  int64_t chunk = ceil_div(ceil_div(pl->kv_limit, target), kBox) * kBox;
  if (pl->paged && chunk > kMaxPagedChunk) chunk = kMaxPagedChunk;
  pl->chunk = static_cast<int>(chunk);
  const int64_t splits = ceil_div(pl->kv_limit, chunk);
  if (splits > (1ll << 31) - 1) return SOLORT_ERR_UNSUPPORTED;
  pl->splits = static_cast<int>(splits);
  pl->rows_total = a->batch * a->q_len * a->num_qo_heads;
  pl->force_partial = force_partial;
  if (pl->splits > 1 || force_partial) {
    pl->part_o_bytes = align_up(static_cast<size_t>(pl->splits) * pl->rows_total * kHD * 4, 256);
    pl->part_lse_bytes = align_up(static_cast<size_t>(pl->splits) * pl->rows_total * 4, 256);
  }
  pl->ws_bytes = pl->part_o_bytes + pl->part_lse_bytes;
  const int bt_ints = pl->paged ? (pl->chunk / a->page_size + 2) : 0;
  // Long splits of at most four query rows run on the tcgen05 kernel, whose tile pipeline streams
  // faster; short splits are latency-bound, where the mma.sync kernel's per-warp tile loop (no
  // cross-warp exchange per tile) finishes first.
  pl->tc = rows <= 4 && pl->chunk >= tc::kMinChunk;
  if (pl->tc) {
    pl->smem_bytes = static_cast<size_t>(tc::kOffBt) + bt_ints * 4;
    if (pl->smem_bytes > static_cast<size_t>(kSmemPerCta)) return SOLORT_ERR_UNSUPPORTED;
    return SOLORT_OK;
  }
  // The block-table slice of a split sits after the ring; a long one costs the ring a stage.
  const int spare = kSmemPerCta - kMaxStages * kStageBytes - kHdrBytes;
  pl->stages = bt_ints * 4 <= spare ? kMaxStages : kMaxStages - 1;
  pl->smem_bytes = static_cast<size_t>(pl->stages) * kStageBytes + kHdrBytes + bt_ints * 4;
  if (pl->smem_bytes > static_cast<size_t>(kSmemPerCta)) return SOLORT_ERR_UNSUPPORTED;
  pl->hold = pl->mt == 1 && (a->flags & SOLORT_DECODE_STABLE_PREFIX) &&
             pl->chunk > kHoldEarlyStages * kTile && pl->chunk <= pl->stages * kTile;
  return SOLORT_OK;
}

inline cudaLaunchConfig_t pdl_config(dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                                     cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

template <int MT, bool PAGED, bool HOLD = false>
int launch_decode(const CUtensorMap& tk, const CUtensorMap& tv, const Params& prm, dim3 grid,
                  size_t smem, cudaStream_t stream) {
  static std::atomic<unsigned> configured{0};  // one bit per device ordinal < 32
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return SOLORT_ERR_CUDA;
  const size_t max_smem = kSmemPerCta;
  if (smem > max_smem) return SOLORT_ERR_UNSUPPORTED;
  if (dev >= 32 || !(configured.load(std::memory_order_acquire) & (1u << dev))) {
    if (cudaFuncSetAttribute(decode_kernel<MT, PAGED, HOLD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(max_smem)) != cudaSuccess ||
        cudaFuncSetAttribute(decode_kernel<MT, PAGED, HOLD>,
                             cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared) != cudaSuccess)
      return SOLORT_ERR_CUDA;
    if (dev < 32) configured.fetch_or(1u << dev, std::memory_order_release);
  }
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_config(grid, dim3(Shape<MT>::kThreads), smem, stream, attr);
  if (cudaLaunchKernelEx(&cfg, decode_kernel<MT, PAGED, HOLD>, tk, tv, prm) != cudaSuccess)
    return SOLORT_ERR_CUDA;
  return launch_status();
}

template <bool PAGED, int RB>
int launch_decode_tc(const CUtensorMap& tk, const CUtensorMap& tv, const Params& prm, dim3 grid,
                     size_t smem, cudaStream_t stream) {
  static std::atomic<unsigned> configured{0};  // one bit per device ordinal < 32
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return SOLORT_ERR_CUDA;
  if (smem > static_cast<size_t>(kSmemPerCta)) return SOLORT_ERR_UNSUPPORTED;
  if (dev >= 32 || !(configured.load(std::memory_order_acquire) & (1u << dev))) {
    if (cudaFuncSetAttribute(decode_tc_kernel<PAGED, RB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kSmemPerCta) != cudaSuccess ||
        cudaFuncSetAttribute(decode_tc_kernel<PAGED, RB>,
                             cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared) != cudaSuccess)
      return SOLORT_ERR_CUDA;
    if (dev < 32) configured.fetch_or(1u << dev, std::memory_order_release);
  }
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_config(grid, dim3(tc::kThreads), smem, stream, attr);
  if (cudaLaunchKernelEx(&cfg, decode_tc_kernel<PAGED, RB>, tk, tv, prm) != cudaSuccess)
    return SOLORT_ERR_CUDA;
  return launch_status();
}

int launch_merge(const MergeParams& mp, cudaStream_t stream) {
  if (mp.rows_total <= 0) return SOLORT_OK;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg =
      pdl_config(dim3(mp.rows_total), dim3(kMergeWarps * 32), 0, stream, attr);
  if (cudaLaunchKernelEx(&cfg, merge_kernel, mp) != cudaSuccess) return SOLORT_ERR_CUDA;
  return launch_status();
}

// The K and V tensor maps of recent calls. An encoding depends only on the base pointers, extents,
// strides and box, which a decode step repeats layer after layer, while encoding costs host time
// on every call; a hit returns the same bytes the encoder would. Direct-mapped, one entry per
// slot, guarded by a mutex (callers may share the library across threads).
struct KvMapEntry {
  bool valid;
  const void* k;
  const void* v;
  uint64_t dims[4];
  uint64_t strides[3];
  uint32_t box[4];
  CUtensorMap tk, tv;
};

int cached_kv_maps(const void* k, const void* v, const uint64_t* dims, const uint64_t* strides,
                   const uint32_t* box, CUtensorMap* tk, CUtensorMap* tv) {
  constexpr int kSlots = 128;
  static std::mutex mu;
  static KvMapEntry cache[kSlots];
  uint64_t h = reinterpret_cast<uintptr_t>(k) ^ (reinterpret_cast<uintptr_t>(v) << 7);
  for (int i = 0; i < 4; ++i) h = h * 1000003u ^ dims[i] ^ (static_cast<uint64_t>(box[i]) << 40);
  for (int i = 0; i < 3; ++i) h = h * 1000003u ^ strides[i];
  KvMapEntry& e = cache[(h ^ (h >> 29)) % kSlots];
  std::lock_guard<std::mutex> lock(mu);
  if (e.valid && e.k == k && e.v == v && !memcmp(e.dims, dims, sizeof(e.dims)) &&
      !memcmp(e.strides, strides, sizeof(e.strides)) && !memcmp(e.box, box, sizeof(e.box))) {
    *tk = e.tk;
    *tv = e.tv;
    return SOLORT_OK;
  }
  int rc = encode_bf16_map(tk, k, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != SOLORT_OK) return rc;
  rc = encode_bf16_map(tv, v, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != SOLORT_OK) return rc;
  e.valid = true;
  e.k = k;
  e.v = v;
  memcpy(e.dims, dims, sizeof(e.dims));
  memcpy(e.strides, strides, sizeof(e.strides));
  memcpy(e.box, box, sizeof(e.box));
  e.tk = *tk;
  e.tv = *tv;
  return SOLORT_OK;
}

int build_kv_maps(const SolortDecodeArgs* a, const Plan& pl, CUtensorMap* tk, CUtensorMap* tv,
                  int* tok_coord, int* box_rows) {
  const int64_t st = a->kv_stride_token, sh = a->kv_stride_head;
  if (st <= 0 || sh <= 0) return SOLORT_ERR_INVALID_ARGUMENT;
  const bool head_inner = sh < st;  // NHD: heads inside a token row
  *tok_coord = head_inner ? 2 : 1;
  uint64_t dims[4], strides[3];
  uint32_t box[4];
  const int nkv = a->num_kv_heads;
  int rows_per_box;
  uint64_t tok_extent;
  if (pl.paged) {
    rows_per_box = a->page_size < kBox ? a->page_size : kBox;
    tok_extent = static_cast<uint64_t>(a->page_size);
  } else {
    rows_per_box = kBox;
    tok_extent = static_cast<uint64_t>(a->kv_capacity);
  }
  *box_rows = rows_per_box;
  dims[0] = kHD;
  box[0] = 64;
  if (head_inner) {
    dims[1] = nkv;
    dims[2] = tok_extent;
    strides[0] = sh * 2;
    strides[1] = st * 2;
    box[1] = 1;
    box[2] = rows_per_box;
  } else {
    dims[1] = tok_extent;
    dims[2] = nkv;
    strides[0] = st * 2;
    strides[1] = sh * 2;
    box[1] = rows_per_box;
    box[2] = 1;
  }
  if (pl.paged) {
    if (a->kv_stride_page <= 0) return SOLORT_ERR_INVALID_ARGUMENT;
    dims[3] = static_cast<uint64_t>(a->num_pages);
    strides[2] = a->kv_stride_page * 2;
  } else {
    dims[3] = 1;
    strides[2] = align_up(strides[1] * dims[2], 16);
  }
  box[3] = 1;
  return cached_kv_maps(a->k, a->v, dims, strides, box, tk, tv);
}

void fill_output_fields(const SolortDecodeArgs* a, Params* prm) {
  prm->out = static_cast<bf16*>(a->out);
  prm->o_sb = a->out_stride_batch;
  prm->o_st = a->out_stride_token;
  prm->o_sh = a->out_stride_head;
  prm->out_f32 = a->lse_out ? a->out_f32 : nullptr;
  prm->lse_out = a->lse_out;
  prm->q_len = a->q_len;
  prm->nh = a->num_qo_heads;
}

}  // namespace dec
}  // namespace solort

using namespace solort;
using namespace solort::dec;

extern "C" int solort_attn_decode_workspace_size(const SolortDecodeArgs* a, size_t* bytes) {
  if (!bytes) return SOLORT_ERR_INVALID_ARGUMENT;
  Plan pl;
  int rc = make_plan(a, &pl);
  if (rc != SOLORT_OK) return rc;
  *bytes = pl.ws_bytes;
  return SOLORT_OK;
}

namespace solort {
namespace dec {

// Shared by solort_attn_decode and solort_attn_decode_exchange (x != nullptr: the merge kernel
// sends every row to the ranks' slots instead of writing an output).
int decode_impl(const SolortDecodeArgs* a, const SolortExchangeArgs* x, void* stream_v) {
  Plan pl;
  int rc = make_plan(a, &pl, x != nullptr);
  if (rc != SOLORT_OK) return rc;
  if (!a->q || !a->k || !a->v || !a->q_pos) return SOLORT_ERR_INVALID_ARGUMENT;
  const bool partial_out = a->lse_out != nullptr;
  if (x) {
    if (a->out || a->out_f32 || a->lse_out || a->q_lens) return SOLORT_ERR_INVALID_ARGUMENT;
    if (x->num_ranks < 1 || x->num_ranks > SOLORT_MAX_RANKS || x->rank < 0 ||
        x->rank >= x->num_ranks)
      return SOLORT_ERR_INVALID_ARGUMENT;
    for (int d = 0; d < x->num_ranks; ++d)
      if (!aligned(x->slot_in_rank[d], 16)) return SOLORT_ERR_INVALID_ARGUMENT;
  } else if (partial_out ? !a->out_f32 : !a->out) {
    return SOLORT_ERR_INVALID_ARGUMENT;
  }
  if (!aligned(a->q, 4) || (a->q_stride_batch | a->q_stride_token | a->q_stride_head) & 1)
    return SOLORT_ERR_INVALID_ARGUMENT;
  if (!x && !partial_out &&
      (!aligned(a->out, 8) || (a->out_stride_batch | a->out_stride_token | a->out_stride_head) & 3))
    return SOLORT_ERR_INVALID_ARGUMENT;
  if (!x && partial_out && (!aligned(a->out_f32, 16) || !aligned(a->lse_out, 4)))
    return SOLORT_ERR_INVALID_ARGUMENT;
  if (pl.paged && (!a->block_table || a->block_table_stride <= 0)) return SOLORT_ERR_INVALID_ARGUMENT;
  if (pl.ws_bytes > 0 &&
      (!a->workspace || a->workspace_bytes < pl.ws_bytes || !aligned(a->workspace, 256)))
    return SOLORT_ERR_WORKSPACE;

  CUtensorMap tk, tv;
  int tok_coord = 1, box_rows = kBox;
  rc = build_kv_maps(a, pl, &tk, &tv, &tok_coord, &box_rows);
  if (rc != SOLORT_OK) return rc;

  Params prm{};
  prm.q = static_cast<const bf16*>(a->q);
  prm.q_sb = a->q_stride_batch;
  prm.q_st = a->q_stride_token;
  prm.q_sh = a->q_stride_head;
  fill_output_fields(a, &prm);
  if (pl.splits > 1 || pl.force_partial) {
    uint8_t* ws = static_cast<uint8_t*>(a->workspace);
    prm.part_o = reinterpret_cast<float*>(ws);
    prm.part_lse = reinterpret_cast<float*>(ws + pl.part_o_bytes);
  }
  prm.q_pos = a->q_pos;
  prm.q_lens = a->q_lens;
  prm.kv_pos_offset = a->kv_pos_offset;
  prm.block_table = a->block_table;
  prm.bt_stride = a->block_table_stride;
  prm.page_size = pl.paged ? a->page_size : 1;
  int shift = 0;
  while (pl.paged && (1 << shift) < a->page_size) ++shift;
  prm.page_shift = shift;
  prm.box_rows = box_rows;
  prm.num_pages = a->num_pages;
  prm.tok_coord = tok_coord;
  prm.kv_limit = pl.kv_limit;
  prm.batch = a->batch;
  prm.nkv = a->num_kv_heads;
  prm.group = a->num_qo_heads / a->num_kv_heads;
  prm.chunk = pl.chunk;
  prm.num_splits = pl.splits;
  prm.stages = pl.stages;
  prm.stable_prefix = (a->flags & SOLORT_DECODE_STABLE_PREFIX) ? 1 : 0;
  prm.force_partial = pl.force_partial ? 1 : 0;
  prm.q_vec16 = aligned(a->q, 16) && ((a->q_stride_batch | a->q_stride_token | a->q_stride_head) & 7) == 0;
  prm.scale_log2 = a->scale * 1.4426950408889634f;

  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  dim3 grid(pl.splits, a->num_kv_heads, a->batch);
  if (pl.tc) {
    rc = pl.paged ? launch_decode_tc<true, 4>(tk, tv, prm, grid, pl.smem_bytes, stream)
                  : launch_decode_tc<false, 4>(tk, tv, prm, grid, pl.smem_bytes, stream);
  } else if (pl.mt == 1) {
    if (pl.hold)
      rc = pl.paged ? launch_decode<1, true, true>(tk, tv, prm, grid, pl.smem_bytes, stream)
                    : launch_decode<1, false, true>(tk, tv, prm, grid, pl.smem_bytes, stream);
    else
      rc = pl.paged ? launch_decode<1, true>(tk, tv, prm, grid, pl.smem_bytes, stream)
                    : launch_decode<1, false>(tk, tv, prm, grid, pl.smem_bytes, stream);
  } else {
    rc = pl.paged ? launch_decode<2, true>(tk, tv, prm, grid, pl.smem_bytes, stream)
                  : launch_decode<2, false>(tk, tv, prm, grid, pl.smem_bytes, stream);
  }
  if (rc != SOLORT_OK || (pl.splits == 1 && !pl.force_partial)) return rc;
  MergeParams mp{};
  mp.o_parts = prm.part_o;
  mp.part_stride = static_cast<int64_t>(pl.rows_total) * kHD;
  mp.lse_parts = prm.part_lse;
  mp.lse_part_stride = pl.rows_total;
  mp.num_parts = pl.splits;
  mp.rows_total = pl.rows_total;
  mp.q_lens = a->q_lens;
  fill_output_fields(a, &mp.out);
  if (x) {
    mp.n_dest = x->num_ranks;
    for (int d = 0; d < x->num_ranks; ++d)
      mp.dest[d] = reinterpret_cast<unsigned long long*>(x->slot_in_rank[d]);
  }
  return launch_merge(mp, stream);
}

}  // namespace dec
}  // namespace solort

extern "C" int solort_attn_decode(const SolortDecodeArgs* a, void* stream) {
  return decode_impl(a, nullptr, stream);
}

extern "C" int solort_attn_decode_exchange_workspace_size(const SolortDecodeArgs* a,
                                                          size_t* bytes) {
  if (!bytes) return SOLORT_ERR_INVALID_ARGUMENT;
  Plan pl;
  int rc = make_plan(a, &pl, true);
  if (rc != SOLORT_OK) return rc;
  *bytes = pl.ws_bytes;
  return SOLORT_OK;
}

extern "C" int solort_attn_decode_exchange(const SolortDecodeArgs* a, const SolortExchangeArgs* x,
                                           void* stream) {
  if (!a || !x) return SOLORT_ERR_INVALID_ARGUMENT;
  return decode_impl(a, x, stream);
}

extern "C" int solort_attn_lse_merge(const SolortMergeArgs* a, void* stream_v) {
  if (!a || !a->o_parts || !a->lse_parts) return SOLORT_ERR_INVALID_ARGUMENT;
  if (a->head_dim != kHD) return SOLORT_ERR_UNSUPPORTED;
  if (a->num_parts <= 0 || a->batch <= 0 || a->q_len <= 0 || a->num_qo_heads <= 0)
    return SOLORT_ERR_INVALID_ARGUMENT;
  if (!aligned(a->o_parts, 16) || (a->part_stride & 3)) return SOLORT_ERR_INVALID_ARGUMENT;
  if (a->out_f32 ? (!a->lse_out || !aligned(a->out_f32, 16)) : !a->out)
    return SOLORT_ERR_INVALID_ARGUMENT;
  if (!a->out_f32 &&
      (!aligned(a->out, 8) || (a->out_stride_batch | a->out_stride_token | a->out_stride_head) & 3))
    return SOLORT_ERR_INVALID_ARGUMENT;
  const int64_t rows = static_cast<int64_t>(a->batch) * a->q_len * a->num_qo_heads;
  if (rows > (1ll << 31) - 1) return SOLORT_ERR_UNSUPPORTED;
  DeviceInfo di;
  int rc = current_device_info(&di);
  if (rc != SOLORT_OK) return rc;
  MergeParams mp{};
  mp.o_parts = a->o_parts;
  mp.part_stride = a->part_stride;
  mp.lse_parts = a->lse_parts;
  mp.lse_part_stride = a->lse_part_stride;
  mp.num_parts = a->num_parts;
  mp.rows_total = static_cast<int>(rows);
  mp.q_lens = nullptr;
  mp.out.out = static_cast<bf16*>(a->out);
  mp.out.o_sb = a->out_stride_batch;
  mp.out.o_st = a->out_stride_token;
  mp.out.o_sh = a->out_stride_head;
  mp.out.out_f32 = a->out_f32;
  mp.out.lse_out = a->lse_out;
  mp.out.q_len = a->q_len;
  mp.out.nh = a->num_qo_heads;
  return launch_merge(mp, static_cast<cudaStream_t>(stream_v));
}

namespace solort {
int read_decode_status(unsigned* flags) {
  unsigned v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_decode_status, sizeof(v)) != cudaSuccess) return SOLORT_ERR_CUDA;
  if (v && cudaMemcpyToSymbol(g_decode_status, &zero, sizeof(zero)) != cudaSuccess)
    return SOLORT_ERR_CUDA;
  *flags |= v;
  return SOLORT_OK;
}
}  // namespace solort

// ------------------------------------------------------------------------------------------
// Allocation-free decode entry point.
//
// Some callers cannot hand this library a workspace: a plugin host whose operator interface passes
// only input and output buffers, or a host runtime that binds this ABI but has no access to a CUDA
// allocator of its own. For them, the split partials live in one file-scope device array, sized
// once for the whole process. Every GPU that loads the library keeps this array until exit, and
// all calls on a GPU share it.
// ------------------------------------------------------------------------------------------
namespace solort {
namespace dec {

constexpr size_t kStaticScratchBytes = size_t(4) << 20;  // 4 MiB of split partials at most
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// Device address of g_static_scratch on the current device. In host code the array's name is only
// a host-side stand-in, so the address is looked up with the device current. The lookup runs on
// every call rather than being cached per device ordinal: once the library's device code is loaded
// it is a table read, and a context that was destroyed and recreated (cudaDeviceReset) may place
// the array elsewhere, which a cached address would miss. The first lookup in a context loads the
// device code, which must not happen inside a stream capture.
int static_scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return SOLORT_ERR_NO_DEVICE;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess || p == nullptr)
    return SOLORT_ERR_CUDA;
  *out = p;
  return SOLORT_OK;
}

}  // namespace dec
}  // namespace solort

extern "C" int solort_attn_decode_static_scratch(const SolortDecodeArgs* a, void* stream) {
  if (!a) return SOLORT_ERR_INVALID_ARGUMENT;
  size_t need = 0;
  int rc = solort_attn_decode_workspace_size(a, &need);
  if (rc != SOLORT_OK) return rc;
  if (need > kStaticScratchBytes) return SOLORT_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  rc = static_scratch_address(&scratch);  // the first call in a device context loads the array
  if (rc != SOLORT_OK) return rc;
  SolortDecodeArgs with_scratch = *a;
  with_scratch.workspace = scratch;
  with_scratch.workspace_bytes = kStaticScratchBytes;
  return solort_attn_decode(&with_scratch, stream);
}
