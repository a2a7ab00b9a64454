// Split-KV GQA decode / verify for sm_100a, static or paged KV, plus the log-sum-exp merge.
//
// One CTA handles one (key split, KV head, sequence). Its KV rows stream through a 3-stage ring
// of 32 KB shared-memory stages (64 tokens of K and V, two 64-dim halves each) filled by TMA tile
// loads with 128-byte swizzle; one elected thread issues them and an mbarrier per stage counts
// the bytes in. Every query row that reads this KV head -- the `group` heads of the group times
// q_len tokens (up to 32 rows) -- is packed into m16 tensor-core tiles, so each K/V byte is read
// from HBM once and from shared memory once for all of them: nothing is expanded with
// repeat_interleave. Four warps take 16-token slices of each stage; QK^T and PV run on mma.sync
// (bf16 in, fp32 accumulate) with an fp32 online softmax in the exp2 domain whose row max is a
// quad shuffle. Warps combine through shared memory at the end; each CTA writes either the final
// bf16 rows (one split) or an fp32 partial (O, LSE) that the merge kernel combines.
//
// Semantics follow the reference's decode (src/solort/model/cuda_graph_executor.py:168,180-184:
// keys 0..pos visible), verify (:250: query i at vpos0+i sees keys <= vpos0+i) and the paged
// addressing of src/solort/cache/kv_cache.py:136-149 (slot = block_table[pos // P] * P + pos % P).
#include <math.h>

#include "common.cuh"
#include "host_util.h"

namespace solort {

__device__ unsigned g_decode_status;

namespace dec {

constexpr int kHD = 128;
constexpr int kTile = 64;                   // tokens per stage
constexpr int kHalfBytes = kTile * 128;     // 64 tokens x 64 dims bf16 (one swizzled box)
constexpr int kKVBytes = 2 * kHalfBytes;    // one of K or V for a stage: 16 KB
constexpr int kStageBytes = 2 * kKVBytes;   // K + V: 32 KB
constexpr int kStages = 3;
constexpr int kThreads = 128;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxChunk = 4096;             // tokens per split at most
constexpr float kLn2 = 0.6931471805599453f;

struct Params {
  const bf16* q;
  int64_t q_sb, q_st, q_sh;
  bf16* out;
  int64_t o_sb, o_st, o_sh;
  float* part_o;    // [S][rows_total][hd]
  float* part_lse;  // [S][rows_total]
  int write_bf16;   // 1: final bf16 rows (single split); 0: fp32 partial rows
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
  float scale_log2;
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

template <int MT, bool PAGED>
__global__ void __launch_bounds__(kThreads, 2)
    decode_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                  const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* stages = align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + kStages * kStageBytes);
  int* abort_flag = reinterpret_cast<int*>(full + kStages);
  int* bt_s = abort_flag + 2;

  const int split = blockIdx.x;
  const int kvh = blockIdx.y;
  const int b = blockIdx.z;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int rows_total = p.batch * p.q_len * p.nh;

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

  // Output row (within all rows) of query row r of this CTA's group.
  auto out_row = [&](int r) { return (b * p.q_len + r / p.group) * p.nh + kvh * p.group + r % p.group; };

  if (ntiles == 0) {
    // Nothing visible in this split: an empty partial (O = 0, LSE = -inf) or, with a single
    // split, zero rows.
    for (int idx = tid; idx < rows_b * (kHD / 4); idx += kThreads) {
      const int r = idx / (kHD / 4), c = (idx % (kHD / 4)) * 4;
      const int qi = r / p.group, h = kvh * p.group + r % p.group;
      if (p.write_bf16) {
        bf16* o = p.out + b * p.o_sb + qi * p.o_st + h * p.o_sh + c;
        *reinterpret_cast<uint2*>(o) = make_uint2(0u, 0u);
      } else {
        const int R = out_row(r);
        float* o = p.part_o + (static_cast<int64_t>(split) * rows_total + R) * kHD + c;
        *reinterpret_cast<float4*>(o) = make_float4(0.f, 0.f, 0.f, 0.f);
        if (c == 0) p.part_lse[static_cast<int64_t>(split) * rows_total + R] = -INFINITY;
      }
    }
    return;
  }

  int lp0 = 0;
  if (PAGED) {
    lp0 = t_begin >> p.page_shift;
    const int lp1 = (t_end - 1) >> p.page_shift;
    for (int i = tid; i <= lp1 - lp0; i += kThreads) bt_s[i] = p.block_table[b * p.bt_stride + lp0 + i];
  }
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    abort_flag[0] = 0;
    fence_mbarrier_init();
  }
  __syncthreads();

  auto issue = [&](int it, int s) {
    uint8_t* Ks = stages + s * kStageBytes;
    uint8_t* Vs = Ks + kKVBytes;
    mbar_arrive_expect_tx(&full[s], kStageBytes);
    const int t0 = t_begin + it * kTile;
    if (!PAGED) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int c1 = p.tok_coord == 1 ? t0 : kvh;
        const int c2 = p.tok_coord == 1 ? kvh : t0;
        tma_load_4d(Ks + h * kHalfBytes, &tmK, &full[s], h * 64, c1, c2, 0);
        tma_load_4d(Vs + h * kHalfBytes, &tmV, &full[s], h * 64, c1, c2, 0);
      }
    } else {
      for (int j = 0; j < kTile; j += p.box_rows) {
        const int tok = t0 + j;
        const int row = tok & (p.page_size - 1);
        // Pages past the split are addressed out of range: TMA fills zeros, reads nothing.
        const int page = tok < t_end ? bt_s[(tok >> p.page_shift) - lp0] : p.num_pages;
        const int c1 = p.tok_coord == 1 ? row : kvh;
        const int c2 = p.tok_coord == 1 ? kvh : row;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          tma_load_4d(Ks + h * kHalfBytes + j * 128, &tmK, &full[s], h * 64, c1, c2, page);
          tma_load_4d(Vs + h * kHalfBytes + j * 128, &tmV, &full[s], h * 64, c1, c2, page);
        }
      }
    }
  };

  if (tid == 0) {
    const int n0 = ntiles < kStages ? ntiles : kStages;
    for (int i = 0; i < n0; ++i) issue(i, i);
  }

  // Query fragments (A operand, m16k16 per (mt, ks)); rows beyond this sequence's rows are zero.
  uint32_t qa[MT][8][4];
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
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = mt * 16 + (lane >> 2) + (e & 1) * 8;
        const int c = ks * 16 + (lane & 3) * 2 + (e >> 1) * 8;
        uint32_t v = 0u;
        if (r < rows_b) {
          const int qi = r / p.group, h = kvh * p.group + r % p.group;
          v = *reinterpret_cast<const uint32_t*>(p.q + b * p.q_sb + qi * p.q_st + h * p.q_sh + c);
        }
        qa[mt][ks][e] = v;
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

  const uint32_t stages_u32 = smem_u32(stages);
  bool ok = true;
  int abort_it = -1;
  for (int it = 0; it < ntiles; ++it) {
    const int s = it % kStages;
    const uint32_t parity = (it / kStages) & 1;
    if (!mbar_wait(&full[s], parity, &g_decode_status)) {
      ok = false;
      abort_flag[0] = 1;
    }
    const int tok0 = t_begin + it * kTile + warp * 16;
    if (ok && tok0 < t_end) {
      const uint32_t Ks = stages_u32 + s * kStageBytes;
      const uint32_t Vs = Ks + kKVBytes;
      if (t_end - tok0 < 16) {
        // Rows past the last key may hold anything (an unfilled page is uninitialised memory);
        // their P is exactly 0, but 0 * NaN is not, so zero this warp's V rows past the end.
        uint8_t* Vg = stages + s * kStageBytes + kKVBytes;
        const int valid = t_end - tok0;
        for (int idx = lane; idx < (16 - valid) * 16; idx += 32) {
          const int trow = warp * 16 + valid + (idx >> 4);
          const int ch = idx & 15;
          *reinterpret_cast<uint4*>(Vg + (ch >> 3) * kHalfBytes + swz128(trow, ch & 7)) =
              make_uint4(0u, 0u, 0u, 0u);
        }
        fence_proxy_async_shared();  // order these writes before the stage's next TMA fill
        __syncwarp();
      }
      float sc[MT][2][4];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) sc[mt][nt][e] = 0.f;
      // S = Q K^T over 128 dims: 8 k-steps, two n8 tiles of tokens.
      {
        const int mi = lane >> 3;
        const int trow = warp * 16 + ((mi >> 1) << 3) + (lane & 7);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const int half = ks >> 2;
          const int chunk = ((ks & 3) << 1) + (mi & 1);
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(b0, b1, b2, b3, Ks + half * kHalfBytes + swz128(trow, chunk));
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            mma_bf16_16816(sc[mt][0], qa[mt][ks], b0, b1);
            mma_bf16_16816(sc[mt][1], qa[mt][ks], b2, b3);
          }
        }
      }
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
              float v = sc[mt][nt][hr * 2 + c] * p.scale_log2;
              v = tok <= lim[mt][hr] ? v : -INFINITY;
              sc[mt][nt][hr * 2 + c] = v;
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
              const float e = exp2f(sc[mt][nt][hr * 2 + c] - ref);
              sc[mt][nt][hr * 2 + c] = e;
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
        pa[mt][0] = pack_bf16x2(sc[mt][0][0], sc[mt][0][1]);
        pa[mt][1] = pack_bf16x2(sc[mt][0][2], sc[mt][0][3]);
        pa[mt][2] = pack_bf16x2(sc[mt][1][0], sc[mt][1][1]);
        pa[mt][3] = pack_bf16x2(sc[mt][1][2], sc[mt][1][3]);
      }
      // O += P V: V^T fragments via ldmatrix.trans, 16 n8 tiles of dims.
      {
        const int mi = lane >> 3;
        const int trow = warp * 16 + ((mi & 1) << 3) + (lane & 7);
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
    __syncthreads();
    if (abort_flag[0]) {
      abort_it = it;
      break;
    }
    if (tid == 0 && it + kStages < ntiles) issue(it + kStages, s);
  }

  if (abort_it >= 0) {
    // A stage never completed within the time limit. Tiles abort_it .. abort_it+kStages-1 may
    // still have copies in flight: give each a bounded wait before the CTA releases its shared
    // memory, and write nothing.
    if (tid == 0) {
      const int last = min(ntiles, abort_it + kStages);
      for (int t = abort_it; t < last; ++t) {
        const uint32_t bar = smem_u32(&full[t % kStages]);
        const uint32_t par = (t / kStages) & 1;
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

  constexpr int kRows = MT * 16;
  float* red = reinterpret_cast<float*>(stages);            // [warps][kRows][hd]
  float* ms = red + kWarps * kRows * kHD;                    // [warps][kRows]
  float* ls = ms + kWarps * kRows;                           // [warps][kRows]
  if ((lane & 3) == 0) {
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const int r = mt * 16 + (lane >> 2) + hr * 8;
        ms[warp * kRows + r] = m_run[mt][hr];
        ls[warp * kRows + r] = l_run[mt][hr];
      }
  }
  __syncthreads();
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int r = mt * 16 + (lane >> 2) + hr * 8;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) M = fmaxf(M, ms[w * kRows + r]);
      const float f = m_run[mt][hr] == -INFINITY ? 0.f : exp2f(m_run[mt][hr] - M);
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        const int c = n * 8 + (lane & 3) * 2;
        float2 v = make_float2(o_acc[mt][n][hr * 2] * f, o_acc[mt][n][hr * 2 + 1] * f);
        *reinterpret_cast<float2*>(red + (warp * kRows + r) * kHD + c) = v;
      }
    }
  __syncthreads();

  for (int idx = tid; idx < rows_b * (kHD / 4); idx += kThreads) {
    const int r = idx / (kHD / 4), c = (idx % (kHD / 4)) * 4;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, ms[w * kRows + r]);
    float L = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float mw = ms[w * kRows + r];
      if (mw != -INFINITY) L += ls[w * kRows + r] * exp2f(mw - M);
      const float4 v = *reinterpret_cast<const float4*>(red + (w * kRows + r) * kHD + c);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    const int qi = r / p.group, h = kvh * p.group + r % p.group;
    if (p.write_bf16) {
      bf16* o = p.out + b * p.o_sb + qi * p.o_st + h * p.o_sh + c;
      uint2 pk;
      pk.x = pack_bf16x2(acc.x * inv, acc.y * inv);
      pk.y = pack_bf16x2(acc.z * inv, acc.w * inv);
      *reinterpret_cast<uint2*>(o) = pk;
    } else {
      const int R = out_row(r);
      float* o = p.part_o + (static_cast<int64_t>(split) * rows_total + R) * kHD + c;
      *reinterpret_cast<float4*>(o) = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
      if (c == 0)
        p.part_lse[static_cast<int64_t>(split) * rows_total + R] =
            L > 0.f ? (M + log2f(L)) * kLn2 : -INFINITY;
    }
  }
}

struct MergeParams {
  const float* o_parts;
  int64_t part_stride;
  const float* lse_parts;
  int64_t lse_part_stride;
  int num_parts;
  int rows_total, q_len, nh;
  bf16* out;
  int64_t o_sb, o_st, o_sh;
  float* out_f32;
  float* lse_out;
  const int32_t* q_lens;  // optional: rows whose token index is past q_lens[b] are skipped
};

// One warp per output row; lane l owns dims 4l..4l+3.
__global__ void __launch_bounds__(128) lse_merge_kernel(const MergeParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int R = blockIdx.x * 4 + warp;
  if (R >= p.rows_total) return;
  if (p.q_lens) {
    const int t = (R / p.nh) % p.q_len, b = R / (p.nh * p.q_len);
    if (t >= p.q_lens[b]) return;
  }
  float mx = -INFINITY;
  for (int i = lane; i < p.num_parts; i += 32) mx = fmaxf(mx, p.lse_parts[i * p.lse_part_stride + R]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float den = 0.f;
  if (mx != -INFINITY) {
    for (int i = 0; i < p.num_parts; ++i) {
      const float l = p.lse_parts[i * p.lse_part_stride + R];
      if (l == -INFINITY) continue;
      const float w = __expf(l - mx);
      den += w;
      const float4 v = *reinterpret_cast<const float4*>(p.o_parts + i * p.part_stride +
                                                        static_cast<int64_t>(R) * kHD + lane * 4);
      acc.x += w * v.x;
      acc.y += w * v.y;
      acc.z += w * v.z;
      acc.w += w * v.w;
    }
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  if (p.out_f32) {
    *reinterpret_cast<float4*>(p.out_f32 + static_cast<int64_t>(R) * kHD + lane * 4) =
        make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
    if (lane == 0) p.lse_out[R] = den > 0.f ? mx + logf(den) : -INFINITY;
  } else {
    const int h = R % p.nh, t = (R / p.nh) % p.q_len, b = R / (p.nh * p.q_len);
    bf16* o = p.out + b * p.o_sb + t * p.o_st + h * p.o_sh + lane * 4;
    uint2 pk;
    pk.x = pack_bf16x2(acc.x * inv, acc.y * inv);
    pk.y = pack_bf16x2(acc.z * inv, acc.w * inv);
    *reinterpret_cast<uint2*>(o) = pk;
  }
}

// ------------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------------

struct Plan {
  int mt = 1;
  bool paged = false;
  int kv_limit = 0;
  int chunk = 0;
  int splits = 0;
  size_t ws_bytes = 0;
  size_t smem_bytes = 0;
  int rows_total = 0;
};

inline int ceil_div(int64_t a, int64_t b) { return static_cast<int>((a + b - 1) / b); }

int make_plan(const SolortDecodeArgs* a, Plan* pl) {
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
  const int resident = 2 * di.sm_count;
  const int heads = a->batch * a->num_kv_heads;
  int target = a->num_splits > 0 ? a->num_splits : (resident / heads > 1 ? resident / heads : 1);
  int chunk = ceil_div(pl->kv_limit, target);
  chunk = ceil_div(chunk, kTile) * kTile;
  if (chunk > kMaxChunk) chunk = kMaxChunk;
  if (chunk < kTile) chunk = kTile;
  pl->chunk = chunk;
  pl->splits = ceil_div(pl->kv_limit, chunk);
  if (pl->splits > 65535 * 16) return SOLORT_ERR_UNSUPPORTED;
  pl->rows_total = a->batch * a->q_len * a->num_qo_heads;
  const bool partial_out = a->lse_out != nullptr;
  if (pl->splits > 1) {
    pl->ws_bytes = align_up(static_cast<size_t>(pl->splits) * pl->rows_total * kHD * 4, 256) +
                   align_up(static_cast<size_t>(pl->splits) * pl->rows_total * 4, 256);
  } else {
    pl->ws_bytes = 0;
  }
  (void)partial_out;
  const int bt_ints = pl->paged ? (chunk / a->page_size + 2) : 0;
  pl->smem_bytes = 1024 + kStages * kStageBytes + kStages * 8 + 8 + bt_ints * 4;
  return SOLORT_OK;
}

template <int MT, bool PAGED>
int launch_decode(const CUtensorMap& tk, const CUtensorMap& tv, const Params& prm, dim3 grid,
                  size_t smem, cudaStream_t stream) {
  static int configured_dev_mask = 0;  // one bit per device ordinal < 31
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 31 && !(configured_dev_mask & (1 << dev))) {
    if (cudaFuncSetAttribute(decode_kernel<MT, PAGED>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             1024 + kStages * kStageBytes + 64 + (kMaxChunk / 8 + 2) * 4) !=
        cudaSuccess)
      return SOLORT_ERR_CUDA;
    configured_dev_mask |= 1 << dev;
  }
  decode_kernel<MT, PAGED><<<grid, kThreads, smem, stream>>>(tk, tv, prm);
  return launch_status();
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
    rows_per_box = a->page_size < kTile ? a->page_size : kTile;
    tok_extent = static_cast<uint64_t>(a->page_size);
  } else {
    rows_per_box = kTile;
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
    const uint64_t s1 = strides[1] * dims[2];
    strides[2] = (s1 + 15) / 16 * 16;
  }
  box[3] = 1;
  int rc = encode_bf16_map(tk, a->k, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != SOLORT_OK) return rc;
  return encode_bf16_map(tv, a->v, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
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

extern "C" int solort_attn_decode(const SolortDecodeArgs* a, void* stream_v) {
  Plan pl;
  int rc = make_plan(a, &pl);
  if (rc != SOLORT_OK) return rc;
  if (!a->q || !a->k || !a->v || !a->q_pos) return SOLORT_ERR_INVALID_ARGUMENT;
  const bool partial_out = a->lse_out != nullptr;
  if (partial_out ? !a->out_f32 : !a->out) return SOLORT_ERR_INVALID_ARGUMENT;
  if (!aligned(a->q, 4) || (a->q_stride_batch | a->q_stride_token | a->q_stride_head) & 1)
    return SOLORT_ERR_INVALID_ARGUMENT;
  if (!partial_out &&
      (!aligned(a->out, 8) || (a->out_stride_batch | a->out_stride_token | a->out_stride_head) & 3))
    return SOLORT_ERR_INVALID_ARGUMENT;
  if (partial_out && (!aligned(a->out_f32, 16) || !aligned(a->lse_out, 4)))
    return SOLORT_ERR_INVALID_ARGUMENT;
  if (pl.paged && (!a->block_table || a->block_table_stride <= 0)) return SOLORT_ERR_INVALID_ARGUMENT;
  if (pl.ws_bytes > 0 && (!a->workspace || a->workspace_bytes < pl.ws_bytes || !aligned(a->workspace, 256)))
    return SOLORT_ERR_WORKSPACE;

  CUtensorMap tk, tv;
  int tok_coord = 1, box_rows = kTile;
  rc = build_kv_maps(a, pl, &tk, &tv, &tok_coord, &box_rows);
  if (rc != SOLORT_OK) return rc;

  Params prm{};
  prm.q = static_cast<const bf16*>(a->q);
  prm.q_sb = a->q_stride_batch;
  prm.q_st = a->q_stride_token;
  prm.q_sh = a->q_stride_head;
  prm.out = static_cast<bf16*>(a->out);
  prm.o_sb = a->out_stride_batch;
  prm.o_st = a->out_stride_token;
  prm.o_sh = a->out_stride_head;
  float* ws_o = nullptr;
  float* ws_l = nullptr;
  if (pl.splits > 1) {
    ws_o = static_cast<float*>(a->workspace);
    ws_l = reinterpret_cast<float*>(static_cast<uint8_t*>(a->workspace) +
                                    align_up(static_cast<size_t>(pl.splits) * pl.rows_total * kHD * 4, 256));
    prm.part_o = ws_o;
    prm.part_lse = ws_l;
    prm.write_bf16 = 0;
  } else if (partial_out) {
    prm.part_o = a->out_f32;
    prm.part_lse = a->lse_out;
    prm.write_bf16 = 0;
  } else {
    prm.write_bf16 = 1;
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
  prm.q_len = a->q_len;
  prm.nh = a->num_qo_heads;
  prm.nkv = a->num_kv_heads;
  prm.group = a->num_qo_heads / a->num_kv_heads;
  prm.chunk = pl.chunk;
  prm.num_splits = pl.splits;
  prm.scale_log2 = a->scale * 1.4426950408889634f;

  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  dim3 grid(pl.splits, a->num_kv_heads, a->batch);
  if (pl.mt == 1) {
    rc = pl.paged ? launch_decode<1, true>(tk, tv, prm, grid, pl.smem_bytes, stream)
                  : launch_decode<1, false>(tk, tv, prm, grid, pl.smem_bytes, stream);
  } else {
    rc = pl.paged ? launch_decode<2, true>(tk, tv, prm, grid, pl.smem_bytes, stream)
                  : launch_decode<2, false>(tk, tv, prm, grid, pl.smem_bytes, stream);
  }
  if (rc != SOLORT_OK) return rc;
  if (pl.splits > 1) {
    MergeParams mp{};
    mp.o_parts = ws_o;
    mp.part_stride = static_cast<int64_t>(pl.rows_total) * kHD;
    mp.lse_parts = ws_l;
    mp.lse_part_stride = pl.rows_total;
    mp.num_parts = pl.splits;
    mp.rows_total = pl.rows_total;
    mp.q_len = a->q_len;
    mp.nh = a->num_qo_heads;
    mp.out = static_cast<bf16*>(a->out);
    mp.o_sb = a->out_stride_batch;
    mp.o_st = a->out_stride_token;
    mp.o_sh = a->out_stride_head;
    mp.out_f32 = partial_out ? a->out_f32 : nullptr;
    mp.lse_out = partial_out ? a->lse_out : nullptr;
    mp.q_lens = a->q_lens;
    lse_merge_kernel<<<ceil_div(pl.rows_total, 4), 128, 0, stream>>>(mp);
    rc = launch_status();
  }
  return rc;
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
  DeviceInfo di;
  int rc = current_device_info(&di);
  if (rc != SOLORT_OK) return rc;
  MergeParams mp{};
  mp.o_parts = a->o_parts;
  mp.part_stride = a->part_stride;
  mp.lse_parts = a->lse_parts;
  mp.lse_part_stride = a->lse_part_stride;
  mp.num_parts = a->num_parts;
  mp.rows_total = a->batch * a->q_len * a->num_qo_heads;
  mp.q_len = a->q_len;
  mp.nh = a->num_qo_heads;
  mp.out = static_cast<bf16*>(a->out);
  mp.o_sb = a->out_stride_batch;
  mp.o_st = a->out_stride_token;
  mp.o_sh = a->out_stride_head;
  mp.out_f32 = a->out_f32;
  mp.lse_out = a->lse_out;
  lse_merge_kernel<<<ceil_div(mp.rows_total, 4), 128, 0, static_cast<cudaStream_t>(stream_v)>>>(mp);
  return launch_status();
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
