// Block-table attention for FEW new rows (a block of decode rows of one or a few requests) on sm_100a.
//
// The twin-tile kernel in attn_sm100.cuh is built for throughput: 256 query rows per CTA, four interleaved chains, KV splits
// merged through fp32 partials in HBM. With one 32-row block per request there are only (sequences x KV heads x 1-2 query
// tiles) units of work; what matters then is how many SMs pull K/V pages at once and how short each CTA's dependent chain
// is. Here:
//   * a CTA owns ONE GQA-packed query tile (<= 128 rows = tokens x heads of a KV group) and a contiguous range of 128-key
//     tiles: Q·K^T (128 x 128) -> softmax -> P·V per tile, S double-buffered in TMEM so the next Q·K^T overlaps the softmax;
//   * the splits of one (sequence, KV head, query tile) form a THREAD-BLOCK CLUSTER (up to 16 CTAs, as many as the device
//     keeps resident), so they are co-scheduled and may meet at a hardware barrier. Every CTA writes its unnormalised O, row
//     maxima and row sums (fp32) to a workspace that stays in L2; after ONE cluster barrier each CTA merges a slice of the
//     head dimension over all shares and writes the final rows. The merge is spread over all CTAs of the unit, there is no
//     second launch and no arrival counter. (Reading the shares straight out of the peers' shared memory was measured
//     slower: 7 us of distributed-shared-memory loads against 2 us through L2 for 10 shares of 64 KB.)
// Operands come by TMA out of the paged pool exactly as in the twin-tile kernel (page id = a tensor-map coordinate, no
// gather); masks follow the same rules (context always visible; new keys block-causal / bidirectional / dense mask / causal).
// Roles: warp 0 TMA producer, warp 1 MMA issuer + TMEM owner, warps 2-5 softmax + epilogue (thread = tile row = TMEM lane).
// Every mbarrier wait is bounded; nobody leaves before the cluster barrier, so a CTA that gave up cannot strand its peers.
#pragma once

#include "attn_sm100.cuh"
#include "gemm_sm100.cuh"

namespace pdllm {
namespace dec {

using tc::mbar_init; using tc::mbar_expect_tx; using tc::mbar_arrive; using tc::mbar_wait; using tc::smem_u32;
using tc::fence_barrier_init; using tc::fence_proxy_async; using tc::tc_fence_before; using tc::tc_fence_after;
using tc::tc_wait_ld; using tc::tc_wait_st; using tc::umma_ss; using tc::umma_ts; using tc::umma_commit;
using tc::desc_kmajor_sw128; using tc::desc_mnmajor_sw128; using tc::make_idesc; using tc::ex2; using tc::TileInfo; using tc::tile_info;
using tc::kTileM; using tc::kTileN; using tc::kHeadDim; using tc::kRescaleThreshold;

constexpr int kThreads = 192;
constexpr int kSoftmaxWarp0 = 2;
constexpr int kQBytes = kTileM * kHeadDim * 2;       // 32 KB: two swizzled [128 rows x 64 cols] halves
constexpr int kKvBytes = kTileN * kHeadDim * 2;      // 32 KB per K or V tile: [column half][128 keys][128 B]
constexpr int kRing = 2;
constexpr int kSmemQ = 0;
constexpr int kSmemK = kQBytes;
constexpr int kSmemV = kSmemK + kRing * kKvBytes;
constexpr int kSmemBar = kSmemV + kRing * kKvBytes;  // 160 KB
constexpr int kSmemBytes = kSmemBar + 256 + 1024;    // + slack to align the base to 1024 B
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;                        // S_0, S_1: 128 fp32 columns each; P (bf16 pairs) aliases the first 64
constexpr uint32_t kColO = 256;                      // O: 128 columns
constexpr int kMaxCluster = 16;
// A CTA's fp32 O share is laid out [column group of 4][128 rows][4]: the 16-byte accesses of a warp (32 consecutive rows, one
// column group) cover 512 contiguous bytes, for the writer and for the merging readers alike.
constexpr int kPartStride = kHeadDim;
constexpr int64_t kShareFloats = static_cast<int64_t>(kTileM) * kPartStride + 2 * kTileM;   // O + (m, l) of one CTA

// Optional timeline of the first CTA (only with -DPDLLM_ENABLE_TRACE): trace[event] = %globaltimer in nanoseconds.
#ifdef PDLLM_ENABLE_TRACE
#define PDLLM_DEC_TRACE(ev) do { if (a.trace != nullptr && blockIdx.x == 0 && (ev) < 64) { long long t_; asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_)); a.trace[(ev)] = t_; } } while (0)
#else
#define PDLLM_DEC_TRACE(ev) do { } while (0)
#endif

// barrier indices
constexpr int kQFull = 0, kKFull = 1, kVFull = 3, kKFree = 5, kVFree = 7, kSFull = 9, kPFull = 11, kPvDone = 13, kNumBars = 15;

struct Args {
  void* out;
  const int32_t* block_table; const int32_t* cu_seqlens_q; const int32_t* seq_lens;
  const uint8_t* mask; int32_t* status;
  long long* trace;    // timeline of CTA 0 in a build with PDLLM_ENABLE_TRACE, else unused
  float* shares;       // [CTA][128 rows][kPartStride] fp32 O, then [CTA][2][128] (m, l)
  int64_t out_stride, block_table_stride, mask_stride_m, mask_stride_n, num_pages;
  int num_seqs, max_pages, num_kv_heads, group, tpt, q_tiles, splits;
  int page_size, has_cache, mask_mode, bidirectional, block_m;
  float scale_log2;
};

template <bool kBf16>
__global__ void __launch_bounds__(kThreads, 1)
attn_decode_sm100_kernel(const __grid_constant__ CUtensorMap q_map, const __grid_constant__ CUtensorMap kn_map,
                         const __grid_constant__ CUtensorMap vn_map, const __grid_constant__ CUtensorMap kc_map,
                         const __grid_constant__ CUtensorMap vc_map, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kSmemBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kSmemBar + 128);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kSmemBar + 136);
  volatile int* tile_flags = reinterpret_cast<volatile int*>(smem + kSmemBar + 144);   // [4]: page of tile (it & 3) was unreadable
  float* part_o = a.shares + static_cast<int64_t>(blockIdx.x) * kShareFloats;     // this CTA's share: O [128 rows][128], then (m, l)
  float* ml = part_o + kTileM * kPartStride;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 64) PDLLM_DEC_TRACE(0);

  // ---- on-chip set-up first: it may run while the previous kernel of the stream is still finishing. Nothing global (the
  // sequence tables, the rows the projections just wrote, the workspace) is touched before grid_dependency_wait().
  if (warp == 0) {
    if (lane == 0) {
      for (int i = 0; i < kNumBars; ++i) mbar_init(&bars[i], (i >= kPFull && i < kPFull + 2) ? 128u : 1u);
      abort_flag[0] = 0;
      fence_barrier_init();
    }
    __syncwarp();
  } else if (warp == 1) {
    gemm::tmem_alloc_cols(tmem_slot, kTmemCols);
  }
  grid_dependency_wait();
  grid_launch_dependents();

  // ---- work unit: (sequence, KV head, query tile) x split; the splits of a unit are the CTAs of one cluster ----
  const int split = static_cast<int>(blockIdx.x) % a.splits;
  int u = static_cast<int>(blockIdx.x) / a.splits;
  const int qt = u % a.q_tiles; u /= a.q_tiles;
  const int kvh = u % a.num_kv_heads;
  const int seq = u / a.num_kv_heads;
  const int q_start = a.cu_seqlens_q[seq];
  const int q_len = a.cu_seqlens_q[seq + 1] - q_start;
  int ctx_len = a.has_cache ? (a.seq_lens[seq] - q_len) : 0;
  if (ctx_len < 0) ctx_len = 0;
  const int G = a.group;
  const int tok0 = qt * a.tpt;
  const int n_tok = min(a.tpt, q_len - tok0);      // <= 0: this query tile does not exist for this sequence
  int new_end = q_len;
  if (n_tok > 0) {
    const int last_m = tok0 + n_tok - 1;
    if (a.mask_mode == PDLLM_MASK_CAUSAL) new_end = min(q_len, last_m + 1);
    else if (!a.bidirectional) new_end = min(q_len, (last_m / a.block_m + 1) * a.block_m);
  }
  const int n_ctx_tiles = (ctx_len + kTileN - 1) / kTileN;
  const int total_tiles = n_ctx_tiles + (new_end + kTileN - 1) / kTileN;
  const int per_split = (total_tiles + a.splits - 1) / a.splits;
  const int t_begin = min(total_tiles, split * per_split);
  const int t_end = min(total_tiles, t_begin + per_split);
  const int n_iter = n_tok > 0 ? t_end - t_begin : 0;

  // ---- the first copies start at once (warp 0) ----
  // one K or V tile of key tile `it` → its ring slot (the caller has made sure the slot is free)
  auto load_kv = [&](int it, int is_v) {
    const int slot = it & 1;
    const TileInfo ti = tile_info(t_begin + it, n_ctx_tiles, ctx_len, new_end);
    uint64_t* bar = &bars[(is_v ? kVFull : kKFull) + slot];
    uint8_t* dst = smem + (is_v ? kSmemV : kSmemK) + slot * kKvBytes;
    mbar_expect_tx(bar, kKvBytes);
    if (ti.is_ctx) {
      const int pidx = ti.key0 / a.page_size;
      const int off = ti.key0 - pidx * a.page_size;
      int page = (pidx < a.max_pages) ? a.block_table[seq * a.block_table_stride + pidx] : -1;
      const bool bad = page < 0 || page >= a.num_pages;
      if (bad) { report_status(a.status, PDLLM_S_BAD_PAGE); page = 0; }   // keep the copy in bounds; the softmax warps hide the tile
      if (!is_v) tile_flags[it & 3] = bad ? 1 : 0;   // reaches the softmax warps through K-full -> S-full; the producer runs at most 3 tiles ahead
      tc::tma_load_5d(is_v ? &vc_map : &kc_map, bar, dst, 0, off, 0, kvh, page);
    } else {
      if (!is_v) tile_flags[it & 3] = 0;
      tc::tma_load_4d(is_v ? &vn_map : &kn_map, bar, dst, 0, q_start + ti.key0, 0, kvh);
    }
  };
  if (warp == 0) {
    if (lane == 0) {
      if (n_iter > 0) {
        mbar_expect_tx(&bars[kQFull], 2u * 64u * 2u * static_cast<uint32_t>(G * a.tpt));
        tc::tma_load_3d(&q_map, &bars[kQFull], smem + kSmemQ, 0, kvh * G, q_start + tok0);
        tc::tma_load_3d(&q_map, &bars[kQFull], smem + kSmemQ + kQBytes / 2, 64, kvh * G, q_start + tok0);
        for (int it = 0; it < n_iter && it < kRing; ++it) { load_kv(it, 0); load_kv(it, 1); }   // both ring slots are free at the start
      }
    }
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x == 64) PDLLM_DEC_TRACE(1);

  if (n_iter > 0) {
    if (warp == 0) {
      // =========================== TMA producer: tiles 2.. as their ring slots come free ===========================
      if (lane == 0) {
        bool ok = true;
        for (int it = kRing; it < n_iter && ok; ++it) {
          const int slot = it & 1;
          const uint32_t use = (it >> 1) & 1;
          for (int is_v = 0; is_v < 2 && ok; ++is_v) {
            ok = mbar_wait(&bars[(is_v ? kVFree : kKFree) + slot], use ^ 1, abort_flag, a);   // the MMAs on tile it - 2 are done
            if (ok) load_kv(it, is_v);
          }
        }
        if (!ok) {   // abandoning: let copies in flight land (bounded)
          const long long t0 = clock64();
          while (clock64() - t0 < 200000) { }
        }
      }
      __syncwarp();
    } else if (warp == 1) {
      // =========================== MMA issuer ===========================
      const uint32_t idesc_qk = make_idesc(kBf16, false, kTileN);     // S[128 x 128 keys] = Q[128 x 128] K^T
      const uint32_t idesc_pv = make_idesc(kBf16, true, kHeadDim);    // O[128 x 128] += P[128 x 128 keys] V
      const uint32_t sq = smem_u32(smem + kSmemQ), sk = smem_u32(smem + kSmemK), sv = smem_u32(smem + kSmemV);
      const uint32_t tO = tmem_base + kColO;
      auto issue_qk = [&](int it) -> bool {
        const int slot = it & 1;
        const uint32_t use = (it >> 1) & 1;
        if (!mbar_wait(&bars[kKFull + slot], use, abort_flag, a)) return false;
        if (!mbar_wait(&bars[kPvDone + slot], use ^ 1, abort_flag, a)) return false;   // S/P buffer (it & 1) is free again
        tc_fence_after();
        if (lane == 0) {
          const uint32_t tS = tmem_base + kColS + slot * kTileN;
#pragma unroll
          for (int kk = 0; kk < kHeadDim / 16; ++kk) {
            const uint32_t qoff = (kk >> 2) * (kQBytes / 2) + (kk & 3) * 32;
            const uint32_t koff = slot * kKvBytes + (kk >> 2) * (kKvBytes / 2) + (kk & 3) * 32;
            umma_ss(tS, desc_kmajor_sw128(sq + qoff), desc_kmajor_sw128(sk + koff), idesc_qk, kk > 0 ? 1u : 0u);
          }
          umma_commit(&bars[kSFull + slot]);
          umma_commit(&bars[kKFree + slot]);
          PDLLM_DEC_TRACE(10 + 4 * it);
        }
        __syncwarp();
        return true;
      };
      bool ok = mbar_wait(&bars[kQFull], 0, abort_flag, a);
      if (ok) ok = issue_qk(0);
      for (int it = 0; it < n_iter && ok; ++it) {
        const int slot = it & 1;
        const uint32_t use = (it >> 1) & 1;
        if (it + 1 < n_iter) { ok = issue_qk(it + 1); if (!ok) break; }
        ok = mbar_wait(&bars[kVFull + slot], use, abort_flag, a);
        if (!ok) break;
        const TileInfo ti = tile_info(t_begin + it, n_ctx_tiles, ctx_len, new_end);
        if (ti.nvalid < kTileN) {
          // rows of V past the last valid key may hold anything (stale page contents); P is 0 there but 0 x NaN is NaN
          for (int i = lane; i < (kTileN - ti.nvalid) * 16; i += 32) {
            const int r = ti.nvalid + (i >> 4), c = i & 15;
            *reinterpret_cast<uint4*>(smem + kSmemV + slot * kKvBytes + (c >> 3) * (kKvBytes / 2) + r * 128 + (c & 7) * 16) = make_uint4(0, 0, 0, 0);
          }
          fence_proxy_async();
          __syncwarp();
        }
        ok = mbar_wait(&bars[kPFull + slot], use, abort_flag, a);
        if (!ok) break;
        tc_fence_after();
        if (lane == 0) {
          const uint32_t tP = tmem_base + kColS + slot * kTileN;
#pragma unroll
          for (int kk = 0; kk < kTileN / 16; ++kk) {
            umma_ts(tO, tP + kk * 8, desc_mnmajor_sw128(sv + slot * kKvBytes + kk * 2048, kKvBytes / 2), idesc_pv, (it > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&bars[kPvDone + slot]);
          umma_commit(&bars[kVFree + slot]);
          PDLLM_DEC_TRACE(11 + 4 * it);
        }
        __syncwarp();
      }
    } else {
      // =========================== softmax (thread = tile row) ===========================
      const int r = (warp & 3) * 32 + lane;
      const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
      const uint32_t tO = tmem_base + lane_base + kColO;
      const int tok_local = r / G;
      const bool row_valid = tok_local < n_tok;
      const int m = tok0 + tok_local;
      int row_new_end = q_len;
      if (a.mask_mode == PDLLM_MASK_CAUSAL) row_new_end = min(q_len, m + 1);
      else if (!a.bidirectional) row_new_end = min(q_len, (m / a.block_m + 1) * a.block_m);
      const bool dense_mask = (a.mask != nullptr) && (a.mask_mode == PDLLM_MASK_BLOCK);
      constexpr uint32_t kNegInf = 0xff800000u;
      constexpr int kHalf = kTileN / 2;
      float m_ref = -INFINITY, l_run = 0.f;
      bool ok = true;
      uint32_t s[kHalf];
      for (int it = 0; it < n_iter && ok; ++it) {
        const int slot = it & 1;
        const uint32_t use = (it >> 1) & 1;
        const TileInfo ti = tile_info(t_begin + it, n_ctx_tiles, ctx_len, new_end);
        int cmax_tile = ti.nvalid;
        if (!ti.is_ctx) cmax_tile = min(cmax_tile, row_new_end - ti.key0);
        const bool use_dense = dense_mask && !ti.is_ctx && row_valid;
        const uint8_t* mrow = use_dense ? a.mask + static_cast<int64_t>(m) * a.mask_stride_m + static_cast<int64_t>(ti.key0) * a.mask_stride_n : nullptr;
        ok = mbar_wait(&bars[kSFull + slot], use, abort_flag, a);
        if (!ok) break;
        tc_fence_after();
        if (threadIdx.x == 64) PDLLM_DEC_TRACE(8 + 4 * it);
        const uint32_t tS = tmem_base + lane_base + kColS + slot * kTileN;
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          tc::tmem_ld32(tS + b * kHalf, s);
          tc::tmem_ld32(tS + b * kHalf + 32, s + 32);
          tc_wait_ld();
          int cmax = cmax_tile - b * kHalf;
          if (tile_flags[it & 3]) cmax = 0;
          if (cmax < kHalf || use_dense) {
#pragma unroll
            for (int j = 0; j < kHalf; ++j) {
              bool vis = j < cmax;
              if (vis && use_dense) vis = mrow[(b * kHalf + j) * a.mask_stride_n] != 0;
              if (!vis) s[j] = kNegInf;
            }
          }
          float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
          for (int j = 0; j < kHalf; j += 4) {
            mx0 = fmaxf(mx0, __uint_as_float(s[j])); mx1 = fmaxf(mx1, __uint_as_float(s[j + 1]));
            mx2 = fmaxf(mx2, __uint_as_float(s[j + 2])); mx3 = fmaxf(mx3, __uint_as_float(s[j + 3]));
          }
          const float m_half = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * a.scale_log2;
          if (it == 0 && b == 0) {
            m_ref = m_half;
          } else {
            const bool grow = m_half > m_ref + kRescaleThreshold;
            if (__any_sync(0xffffffffu, grow)) {
              // O must hold every product issued so far: the previous tile's P·V may still be in flight
              if (it > 0) {
                ok = mbar_wait(&bars[kPvDone + ((it - 1) & 1)], ((it - 1) >> 1) & 1, abort_flag, a);
                if (!ok) break;
                tc_fence_after();
              }
              const float m_new = grow ? m_half : m_ref;
              const float alpha = grow ? ex2(m_ref - m_new) : 1.f;
              l_run *= alpha;
              if (it > 0) {
                uint32_t o[16];
#pragma unroll 1
                for (int c = 0; c < kHeadDim / 16; ++c) {
                  tc::tmem_ld16(tO + c * 16, o);
                  tc_wait_ld();
#pragma unroll
                  for (int j = 0; j < 16; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * alpha);
                  tc::tmem_st16(tO + c * 16, o);
                }
                tc_wait_st();
              }
              m_ref = m_new;
            }
          }
          const float m_use = (m_ref == -INFINITY) ? 0.f : m_ref;
          float l0 = 0.f, l1 = 0.f, l2 = 0.f, l3 = 0.f;
          uint32_t packed[kHalf / 2];
#pragma unroll
          for (int j = 0; j < kHalf; j += 4) {
            const float p0 = ex2(fmaf(__uint_as_float(s[j]), a.scale_log2, -m_use));
            const float p1 = ex2(fmaf(__uint_as_float(s[j + 1]), a.scale_log2, -m_use));
            const float p2 = ex2(fmaf(__uint_as_float(s[j + 2]), a.scale_log2, -m_use));
            const float p3 = ex2(fmaf(__uint_as_float(s[j + 3]), a.scale_log2, -m_use));
            l0 += p0; l1 += p1; l2 += p2; l3 += p3;
            if (kBf16) {
              __nv_bfloat162 h0 = __floats2bfloat162_rn(p0, p1), h1 = __floats2bfloat162_rn(p2, p3);
              packed[j >> 1] = *reinterpret_cast<uint32_t*>(&h0);
              packed[(j >> 1) + 1] = *reinterpret_cast<uint32_t*>(&h1);
            } else {
              __half2 h0 = __floats2half2_rn(p0, p1), h1 = __floats2half2_rn(p2, p3);
              packed[j >> 1] = *reinterpret_cast<uint32_t*>(&h0);
              packed[(j >> 1) + 1] = *reinterpret_cast<uint32_t*>(&h1);
            }
          }
          // P of half b: 64 keys = 32 packed columns at [b * 32, b * 32 + 32) of this S buffer; half 1 of S (columns 64..127)
          // is only overwritten by nothing, half 0 (already in registers) by both
          tc::tmem_st32(tS + b * (kHalf / 2), packed);
          l_run += (l0 + l1) + (l2 + l3);
        }
        if (!ok) break;
        tc_wait_st();
        tc_fence_before();
        mbar_arrive(&bars[kPFull + slot]);
        if (threadIdx.x == 64) PDLLM_DEC_TRACE(9 + 4 * it);
      }
      // ---- this CTA's result: O (unnormalised, relative to m_ref), m_ref, l_run ----
      if (ok) ok = mbar_wait(&bars[kPvDone + ((n_iter - 1) & 1)], ((n_iter - 1) >> 1) & 1, abort_flag, a);
      if (threadIdx.x == 64) PDLLM_DEC_TRACE(2);
      if (ok) {
        tc_fence_after();
        if (a.splits == 1) {
          const float inv = (l_run > 0.f) ? 1.f / l_run : 0.f;
          const int head_local = r - tok_local * G;
          uint8_t* out_row = reinterpret_cast<uint8_t*>(a.out) +
                             ((static_cast<int64_t>(q_start + m)) * a.out_stride + static_cast<int64_t>(kvh * G + head_local) * kHeadDim) * 2;
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tc::tmem_ld32(tO + c * 32, o);
            tc_wait_ld();
            if (row_valid) {
              uint32_t pk[16];
#pragma unroll
              for (int j = 0; j < 32; j += 2) {
                const float o0 = __uint_as_float(o[j]) * inv, o1 = __uint_as_float(o[j + 1]) * inv;
                if (kBf16) { __nv_bfloat162 h = __floats2bfloat162_rn(o0, o1); pk[j >> 1] = *reinterpret_cast<uint32_t*>(&h); }
                else { __half2 h = __floats2half2_rn(o0, o1); pk[j >> 1] = *reinterpret_cast<uint32_t*>(&h); }
              }
              uint4* dst = reinterpret_cast<uint4*>(out_row + c * 64);
#pragma unroll
              for (int j = 0; j < 4; ++j) dst[j] = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
            }
          }
        } else {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tc::tmem_ld32(tO + c * 32, o);
            tc_wait_ld();
#pragma unroll
            for (int j = 0; j < 8; ++j)
              *reinterpret_cast<uint4*>(part_o + (static_cast<int64_t>(c * 8 + j) * kTileM + r) * 4) = make_uint4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
          }
          ml[r] = m_ref;
          ml[kTileM + r] = l_run;
        }
      } else if (a.splits > 1) {
        ml[r] = -INFINITY; ml[kTileM + r] = 0.f;      // abandoned: a neutral share (the launch is flagged invalid anyway)
      }
    }
  } else if (a.splits > 1 && warp >= kSoftmaxWarp0) {
    // nothing to attend in this split (or no such query tile): a neutral share
    const int r = (warp & 3) * 32 + lane;
    ml[r] = -INFINITY; ml[kTileM + r] = 0.f;
  }

  // ---- merge across the cluster: CTA of rank p finishes a slice of the head dimension for every row ----
  if (a.splits > 1) {
    __threadfence();                    // this CTA's share is visible device-wide before it arrives
    __syncwarp();
    if (threadIdx.x == 64) PDLLM_DEC_TRACE(3);
    gemm::cluster_sync_all();
    if (threadIdx.x == 64) PDLLM_DEC_TRACE(4);
    if (warp >= kSoftmaxWarp0 && n_tok > 0) {
      const int r = (warp & 3) * 32 + lane;
      const int tok_local = r / G;
      if (tok_local < n_tok) {
        const int S = a.splits;
        const int rank = static_cast<int>(gemm::cluster_ctarank());
        const int cols = (kHeadDim / 8 + S - 1) / S * 8;          // a multiple of 8 columns (16 bytes of output) per rank
        const int d0 = rank * cols, d1 = min(kHeadDim, d0 + cols);
        if (d0 < d1) {
          const float* unit_shares = a.shares + static_cast<int64_t>(blockIdx.x - rank) * kShareFloats;   // share of rank 0 of this cluster
          // all loads of a batch are issued before the first value is used
          float w[kMaxCluster], lsum[kMaxCluster];
#pragma unroll
          for (int p = 0; p < kMaxCluster; ++p) {
            const float* pml = unit_shares + p * kShareFloats + kTileM * kPartStride;
            w[p] = p < S ? __ldcg(pml + r) : -INFINITY;
            lsum[p] = p < S ? __ldcg(pml + kTileM + r) : 0.f;
          }
          float M = -INFINITY;
#pragma unroll
          for (int p = 0; p < kMaxCluster; ++p) M = fmaxf(M, w[p]);
          float denom = 0.f;
#pragma unroll
          for (int p = 0; p < kMaxCluster; ++p) {
            w[p] = (w[p] == -INFINITY) ? 0.f : exp2f(w[p] - M);
            denom += w[p] * lsum[p];
          }
          const float inv = denom > 0.f ? 1.f / denom : 0.f;
          const int head_local = r - tok_local * G;
          uint8_t* out_row = reinterpret_cast<uint8_t*>(a.out) +
                             ((static_cast<int64_t>(q_start + tok0 + tok_local)) * a.out_stride + static_cast<int64_t>(kvh * G + head_local) * kHeadDim) * 2;
          // Every share's slice of this row is requested before the first value is used: one L2 round trip per batch of 8
          // shares instead of one per share. kCols4 16-byte loads per share: 2 when a cluster of 16 leaves 8 columns per
          // rank, 4 for clusters of 8 to 15, 8 below.
          auto merge_cols = [&](auto kCols4Tag, int d0) {          // columns [d0, min(d1, d0 + 4 kCols4))
            constexpr int kCols4 = decltype(kCols4Tag)::value;
            float acc[4 * kCols4];
#pragma unroll
            for (int j = 0; j < 4 * kCols4; ++j) acc[j] = 0.f;
            const float* first = unit_shares + (static_cast<int64_t>(d0 / 4) * kTileM + r) * 4;
            constexpr int kBatch = kCols4 >= 8 ? 4 : 8;
#pragma unroll 1
            for (int pb = 0; pb < S; pb += kBatch) {                // rank order: the result does not depend on timing
              float4 v[kBatch][kCols4];
#pragma unroll
              for (int q = 0; q < kBatch; ++q) {
                const int p = pb + q;
                const bool live = p < S && w[p] != 0.f;             // a neutral share has no O behind it
                const float4* src = reinterpret_cast<const float4*>(first + p * kShareFloats);
#pragma unroll
                for (int c = 0; c < kCols4; ++c) v[q][c] = (live && d0 + 4 * c < d1) ? __ldcg(src + c * kTileM) : make_float4(0.f, 0.f, 0.f, 0.f);
              }
#pragma unroll
              for (int q = 0; q < kBatch; ++q) {
                const float wp = (pb + q) < S ? w[pb + q] : 0.f;
#pragma unroll
                for (int c = 0; c < kCols4; ++c) {
                  acc[4 * c] = fmaf(wp, v[q][c].x, acc[4 * c]); acc[4 * c + 1] = fmaf(wp, v[q][c].y, acc[4 * c + 1]);
                  acc[4 * c + 2] = fmaf(wp, v[q][c].z, acc[4 * c + 2]); acc[4 * c + 3] = fmaf(wp, v[q][c].w, acc[4 * c + 3]);
                }
              }
            }
#pragma unroll
            for (int c = 0; c < kCols4; c += 2) {
              if (d0 + 4 * c >= d1) break;
              uint32_t pk[4];
#pragma unroll
              for (int j = 0; j < 8; j += 2) {
                const float x0 = acc[4 * c + j] * inv, x1 = acc[4 * c + j + 1] * inv;
                if (kBf16) { __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1); pk[j >> 1] = *reinterpret_cast<uint32_t*>(&h); }
                else { __half2 h = __floats2half2_rn(x0, x1); pk[j >> 1] = *reinterpret_cast<uint32_t*>(&h); }
              }
              *reinterpret_cast<uint4*>(out_row + (d0 + 4 * c) * 2) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            }
          };
          if (cols <= 8) merge_cols(std::integral_constant<int, 2>(), d0);
          else if (cols <= 16) merge_cols(std::integral_constant<int, 4>(), d0);
          else {
            for (int dd = d0; dd < d1; dd += 32) merge_cols(std::integral_constant<int, 8>(), dd);   // clusters of 2 to 7
          }
        }
      }
    }
    if (threadIdx.x == 64) PDLLM_DEC_TRACE(5);
  }

  // ---- teardown ----
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tc::tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---- host side ---------------------------------------------------------------------------------------------
struct Plan {
  bool use;          // this kernel serves the shape
  int group, tpt, q_tiles, splits;
  int64_t units;
};

inline Plan make_plan(const pdllm_attn_params* p) {
  Plan pl;
  pl.group = p->num_q_heads / p->num_kv_heads;
  pl.tpt = kTileM / pl.group;
  pl.q_tiles = (p->max_query_len + pl.tpt - 1) / pl.tpt;
  if (pl.q_tiles < 1) pl.q_tiles = 1;
  pl.units = static_cast<int64_t>(p->num_seqs) * p->num_kv_heads * pl.q_tiles;
  const int sms = sm_count();
  const int key_tiles = (p->max_seq_len + kTileN - 1) / kTileN + 1;
  // Few units and enough keys to split: otherwise the twin-tile kernel (whole waves of units, K/V shared by two query
  // tiles) is the better tool. Splits: as many as fill the SMs, at least two key tiles each, at most a cluster.
  int64_t splits = pl.units > 0 ? sms / pl.units : 1;
  if (splits > kMaxCluster) splits = kMaxCluster;
  if (splits > key_tiles / 2) splits = key_tiles / 2;
  pl.use = pl.units > 0 && 2 * pl.units <= sms && splits >= 2 && p->num_splits <= 0;
  pl.splits = static_cast<int>(splits < 1 ? 1 : splits);
  return pl;
}

// one share per CTA of the largest grid the plan may launch
// (behind the header of arrival counters that the twin-tile kernel keeps zeroed at the start of the same workspace)
inline int64_t workspace_bytes(const Plan& pl) { return tc::kCounterHeaderBytes + pl.units * pl.splits * kShareFloats * 4; }

inline int launch(const pdllm_attn_params* p, const Plan& pl, cudaStream_t stream) {
  if (p->workspace == nullptr || p->workspace_bytes < workspace_bytes(pl))
    return fail(PDLLM_E_WORKSPACE, "attention (few rows) needs %lld workspace bytes, got %lld", static_cast<long long>(workspace_bytes(pl)),
                static_cast<long long>(p->workspace_bytes));
  const bool bf16 = p->dtype == PDLLM_BF16;
  const bool has_cache = p->kv_layout == PDLLM_KV_UNIFIED && p->k_cache != nullptr && p->num_pages > 0;
  CUtensorMap q_map, kn_map, vn_map, kc_map, vc_map;
  int rc;
  {
    uint64_t dims[3] = {static_cast<uint64_t>(kHeadDim), static_cast<uint64_t>(p->num_q_heads), static_cast<uint64_t>(p->total_q)};
    uint64_t str[2] = {static_cast<uint64_t>(kHeadDim) * 2, static_cast<uint64_t>(p->q_stride) * 2};
    uint32_t box[3] = {64, static_cast<uint32_t>(pl.group), static_cast<uint32_t>(pl.tpt)};
    if ((rc = tc::encode_map(&q_map, bf16, p->q, 3, dims, str, box)) != 0) return rc;
  }
  {
    // new K/V rows [T, Hkv, D] seen as (64 cols, T rows, 2 column halves, Hkv): one box = [2][128 rows][64 cols]
    uint64_t dims[4] = {64, static_cast<uint64_t>(p->total_q), 2, static_cast<uint64_t>(p->num_kv_heads)};
    uint32_t box[4] = {64, kTileN, 2, 1};
    uint64_t strk[3] = {static_cast<uint64_t>(p->k_stride) * 2, 128, static_cast<uint64_t>(kHeadDim) * 2};
    uint64_t strv[3] = {static_cast<uint64_t>(p->v_stride) * 2, 128, static_cast<uint64_t>(kHeadDim) * 2};
    if ((rc = tc::encode_map(&kn_map, bf16, p->k_new, 4, dims, strk, box)) != 0) return rc;
    if ((rc = tc::encode_map(&vn_map, bf16, p->v_new, 4, dims, strv, box)) != 0) return rc;
  }
  if (has_cache) {
    const uint64_t row = static_cast<uint64_t>(kHeadDim) * 2 * p->num_kv_heads;
    uint64_t dims[5] = {64, static_cast<uint64_t>(p->page_size), 2, static_cast<uint64_t>(p->num_kv_heads), static_cast<uint64_t>(p->num_pages)};
    uint64_t str[4] = {row, 128, static_cast<uint64_t>(kHeadDim) * 2, row * p->page_size};
    uint32_t box[5] = {64, kTileN, 2, 1, 1};
    if ((rc = tc::encode_map(&kc_map, bf16, p->k_cache, 5, dims, str, box)) != 0) return rc;
    if ((rc = tc::encode_map(&vc_map, bf16, p->v_cache, 5, dims, str, box)) != 0) return rc;
  } else {
    kc_map = kn_map; vc_map = vn_map;
  }
  Args a;
  a.out = p->out; a.block_table = p->block_table; a.cu_seqlens_q = p->cu_seqlens_q; a.seq_lens = p->seq_lens;
  a.mask = p->mask; a.status = p->status; a.trace = reinterpret_cast<long long*>(p->trace);
  a.shares = reinterpret_cast<float*>(static_cast<char*>(p->workspace) + tc::kCounterHeaderBytes);
  a.out_stride = p->out_stride; a.block_table_stride = p->block_table_stride;
  a.mask_stride_m = p->mask_stride_m; a.mask_stride_n = p->mask_stride_n; a.num_pages = has_cache ? p->num_pages : 0;
  a.num_seqs = p->num_seqs; a.max_pages = p->max_pages; a.num_kv_heads = p->num_kv_heads;
  a.group = pl.group; a.tpt = pl.tpt; a.q_tiles = pl.q_tiles; a.splits = pl.splits;
  a.page_size = p->page_size > 0 ? p->page_size : kTileN; a.has_cache = has_cache ? 1 : 0;
  a.mask_mode = p->mask_mode; a.bidirectional = p->bidirectional;
  a.block_m = 2 * (p->diffusion_blk > 0 ? p->diffusion_blk : 32);
  a.scale_log2 = p->sm_scale * 1.4426950408889634f;

  auto* fn = bf16 ? attn_decode_sm100_kernel<true> : attn_decode_sm100_kernel<false>;
  static std::mutex mu;
  static bool done[64] = {false};
  static int fits[64][kMaxCluster + 1] = {};     // per device and cluster size: resident clusters + 1 (0 = not asked yet)
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 0 || dev >= 64 || !done[dev]) {
      for (auto* f : {attn_decode_sm100_kernel<true>, attn_decode_sm100_kernel<false>}) {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(f, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);   // clusters of up to 16
        if (e != cudaSuccess) return fail(static_cast<int>(e), "cudaFuncSetAttribute(attn_decode): %s", cudaGetErrorString(e));
      }
      if (dev >= 0 && dev < 64) done[dev] = true;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;   // see launch_dependent(): start ahead of the predecessor's end
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // every cluster of the launch should be resident at once: the largest cluster size, from the planned one down, that fits
  int splits = pl.splits;
  for (; splits >= 2; --splits) {
    int n_fit = -1;
    {
      std::lock_guard<std::mutex> lock(mu);
      if (dev >= 0 && dev < 64 && fits[dev][splits] > 0) n_fit = fits[dev][splits] - 1;
    }
    if (n_fit < 0) {
      cfg.gridDim = dim3(static_cast<unsigned>(pl.units * splits), 1, 1);
      attr[0].val.clusterDim.x = static_cast<unsigned>(splits);
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess) { (void)cudaGetLastError(); n = 0; }
      n_fit = n;
      std::lock_guard<std::mutex> lock(mu);
      if (dev >= 0 && dev < 64) fits[dev][splits] = n + 1;
    }
    if (n_fit >= pl.units) break;
  }
  if (splits < 2) return PDLLM_E_UNSUPPORTED;      // no cluster fits: the caller falls back to the twin-tile kernel
  a.splits = splits;
  cfg.gridDim = dim3(static_cast<unsigned>(pl.units * splits), 1, 1);
  attr[0].val.clusterDim.x = static_cast<unsigned>(splits);
  cfg.numAttrs = dependent_launch_enabled() ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, fn, q_map, kn_map, vn_map, kc_map, vc_map, a);
  if (e != cudaSuccess) return fail(static_cast<int>(e), "attn_decode_sm100_kernel (clusters of %d): %s", splits, cudaGetErrorString(e));
  return check_launch("attn_decode_sm100_kernel");
}

}  // namespace dec
}  // namespace pdllm
