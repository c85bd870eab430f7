// Block-table attention on the 5th-generation tensor cores (sm_100a): tcgen05.mma with TMEM accumulators,
// operands staged by TMA straight out of the paged pool (no gather), online softmax in registers.
//
// Work unit (one CTA, one per SM): TWO GQA-packed query tiles of one (sequence, KV head) x one contiguous range
// of 128-key tiles.
//   * query tile  = up to 128 rows = tpt tokens x G query heads of one KV group (row = token*G + head), so the
//     K/V pages of a KV head are read once for all G heads that share it, and once for both query tiles;
//   * key tiles   = the sequence's selected prefix pages in block-table order (any physical order), then the new
//     rows themselves; a KV split assigns each CTA a sub-range; the CTA that finishes a query-tile pair last merges the partials.
// Every key tile is processed as two 64-key halves b, so four chains (query tile X) x (half b) run interleaved:
// while the softmax warps of X work on S_Xb, the tensor core computes P·V and the next Q·K of the other chains.
// Roles: warps 0-3 softmax + epilogue of query tile A, warps 4-7 of query tile B (thread r owns tile row r = TMEM
// lane r), warp 8 TMA producer + TMEM allocator, warps 9-12 MMA issuers (one per chain). TMEM (all 512 columns): S_A0 S_A1 S_B0 S_B1
// (64 fp32 columns each; P, bf16 pairs, aliases the first 32) and O_A, O_B (128 columns each). Shared memory:
// Q_A, Q_B 32 KB each, and two rings of four 16 KB slots for K and V half-tiles, all in the 128-byte-swizzled
// layouts that TMA writes and the MMA descriptors read; the rings keep three copies in flight per operand,
// which covers the ~2000-cycle latency of a TMA copy.
// Every mbarrier wait is bounded; on expiry the CTA raises PDLLM_S_WAIT_TIMEOUT, drains and frees its TMEM.
#pragma once

#include <cuda.h>

#include <mutex>
#include <vector>

#include "common.cuh"

namespace pdllm {
namespace tc {

constexpr int kTileM = 128;
constexpr int kTileN = 128;
constexpr int kHeadDim = 128;
constexpr int kHalfN = kTileN / 2;                  // keys per S buffer
constexpr int kThreads = 416;                       // warps 0-7 softmax (two query tiles), warp 8 producer, warps 9-12 MMA issuers
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp0 = 9;                       // one issuer warp per chain (query tile, key half)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;                       // S_A0, S_A1, S_B0, S_B1: 64 columns each (P aliases the first 32)
constexpr uint32_t kColO = 256;                     // O_A, O_B: 128 columns each
constexpr int kHalfBytes = kTileM * 64 * 2;         // one [128 rows x 64 cols] swizzled half of a Q tile = 16 KB
constexpr int kTileBytes = 2 * kHalfBytes;          // 32 KB per Q tile
constexpr int kSlotBytes = kHalfN * kHeadDim * 2;   // one K_b or V_b slot: [2 halves of the head dim][64 keys][128 B] = 16 KB
constexpr int kRing = 4;                            // slots per ring (K and V each): copies run up to 3 half-tiles ahead
constexpr int kSmemQ = 0;
constexpr int kSmemK = 2 * kTileBytes;
constexpr int kSmemV = kSmemK + kRing * kSlotBytes;
constexpr int kSmemBar = kSmemV + kRing * kSlotBytes;
constexpr int kSmemBytes = kSmemBar + 512 + 1024;   // + barriers/flags + slack to align the base to 1024 B
constexpr long long kWaitLimitCycles = 1ll << 31;   // about a second
constexpr float kRescaleThreshold = 8.0f;           // log2 units: rescale O only when the row max grew by > 2^8

// barrier indices
constexpr int kQFull = 0;
constexpr int kKFull = 1;              // [kRing]
constexpr int kVFull = kKFull + kRing; // [kRing]
constexpr int kSFull = kVFull + kRing; // [query tile][half] = 4
constexpr int kPFull = kSFull + 4;     // 4, 128 arrivals each
constexpr int kPvDone = kPFull + 4;    // 4
constexpr int kKFree = kPvDone + 4;    // [kRing], one arrival per active query tile: every Q·K on the slot is done
constexpr int kVFree = kKFree + kRing; // [kRing], likewise for P·V
constexpr int kNumBars = kVFree + kRing;

struct Args {
  void* out;
  const int32_t* block_table; const int32_t* cu_seqlens_q; const int32_t* seq_lens;
  const uint8_t* mask; int32_t* status;
  long long* trace;                // optional pipeline timestamps, see trace_event
  float* part_o; float* part_ml;   // split-KV partials: O as [unit][D][128], (m, l) as [unit][2][128]
  int* split_arrivals;             // [seq][kv head][query-tile pair]: splits finished so far (zeroed before the launch)
  int64_t out_stride, block_table_stride, mask_stride_m, mask_stride_n, num_pages;
  int num_seqs, max_pages, num_q_heads, num_kv_heads, group, tpt, q_tiles, q_pairs, num_splits;
  int first_permille;  // uneven two-way split: share (in 1/1000) of a unit's key tiles that split 0 takes; 0 = even splits
  int base_ctas;       // (sequence, KV head, query-tile pair) units
  int n_whole;         // the first n_whole units run unsplit in CTAs [0, n_whole), ahead of the others' splits:
                       // blockIdx = n_whole + split * (base_ctas - n_whole) + (unit - n_whole)
  int tile0;           // first query tile of unit n_whole: partials exist for query tiles >= tile0 only
  int fused_merge;     // 1: the last CTA of a tile pair merges the splits; 0: attn_combine_kernel does, after this kernel
  int page_size, has_cache, mask_mode, bidirectional, block_m, is_bf16;
  float scale_log2;  // sm_scale * log2(e)
};

// ---- PTX wrappers ---------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}
// Bounded wait. Returns false when another role already gave up or when the limit expired.
template <bool kBackoff = false, class ArgsT>
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, const ArgsT& a) {
  if (mbar_try_wait(bar, parity)) return true;
  long long t0 = clock64();
  uint32_t spins = 0;
  while (!mbar_try_wait(bar, parity)) {
    // the producer and MMA warps share their scheduler with a softmax warp: sleep between polls instead of
    // competing with it for issue slots
    if (kBackoff) __nanosleep(40);
    if (((++spins) & 0x3f) == 0) {
      if (*abort_flag) return false;
      if (clock64() - t0 > kWaitLimitCycles) {
        *abort_flag = 1;
        // low byte: the status code; above it, for diagnosis: barrier index in the CTA's barrier array, warp, parity
        const int which = static_cast<int>((smem_u32(bar) & 0x3ff) >> 3);
        const int code = PDLLM_S_WAIT_TIMEOUT | (which << 8) | ((threadIdx.x >> 5) << 16) | (parity << 24);
        report_status(a.status, code);
#ifdef PDLLM_ENABLE_TRACE
        if (a.trace != nullptr && (threadIdx.x & 31) == 0) a.trace[8 * 64 * 16 - 64 + (threadIdx.x >> 5)] = code;  // per-warp record
#endif
        return false;
      }
    }
  }
  return true;
}

__device__ __forceinline__ void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tma_load_3d(const CUtensorMap* map, uint64_t* bar, void* dst, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d(const CUtensorMap* map, uint64_t* bar, void* dst, int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void tma_load_5d(const CUtensorMap* map, uint64_t* bar, void* dst, int c0, int c1, int c2, int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6, %7}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)), "r"(cols) : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}
// mbarrier arrives once every tcgen05 operation issued so far by this thread has completed
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

#define PDLLM_R32(a, o) \
  "=r"(a[o + 0]), "=r"(a[o + 1]), "=r"(a[o + 2]), "=r"(a[o + 3]), "=r"(a[o + 4]), "=r"(a[o + 5]), "=r"(a[o + 6]), "=r"(a[o + 7]), \
  "=r"(a[o + 8]), "=r"(a[o + 9]), "=r"(a[o + 10]), "=r"(a[o + 11]), "=r"(a[o + 12]), "=r"(a[o + 13]), "=r"(a[o + 14]), "=r"(a[o + 15])
#define PDLLM_W16(a, o) \
  "r"(a[o + 0]), "r"(a[o + 1]), "r"(a[o + 2]), "r"(a[o + 3]), "r"(a[o + 4]), "r"(a[o + 5]), "r"(a[o + 6]), "r"(a[o + 7]), \
  "r"(a[o + 8]), "r"(a[o + 9]), "r"(a[o + 10]), "r"(a[o + 11]), "r"(a[o + 12]), "r"(a[o + 13]), "r"(a[o + 14]), "r"(a[o + 15])

// 32 lanes x 32 consecutive 32-bit columns: thread t reads lane (base + t), registers = columns
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : PDLLM_R32(r, 0), PDLLM_R32(r, 16)
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
      ::"r"(taddr), PDLLM_W16(r, 0), PDLLM_W16(r, 16)
      : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : PDLLM_R32(r, 0)
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};"
      ::"r"(taddr), PDLLM_W16(r, 0)
      : "memory");
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---- shared-memory matrix descriptors (version 1 = Blackwell, 128-byte swizzle) -----------------------------
// K-major operand: rows of 64 elements (128 B), 8-row swizzle atoms stacked 1024 B apart.
__device__ __forceinline__ uint64_t desc_kmajor_sw128(uint32_t saddr) {
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}
// MN-major operand (V as B of P*V): 64 contiguous N elements per row, 8 K-rows per atom (1024 B apart along K),
// second 64-element N group `lbo_bytes` away.
__device__ __forceinline__ uint64_t desc_mnmajor_sw128(uint32_t saddr, uint32_t lbo_bytes) {
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(lbo_bytes >> 4) << 16) | (64ull << 32) |
         (1ull << 46) | (2ull << 61);
}
// instruction descriptor, kind::f16: fp32 accumulate, A/B bf16 (1) or fp16 (0), M=128, N=128
__host__ __device__ constexpr uint32_t make_idesc(bool bf16, bool b_mn_major, int n) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(n >> 3) << 17) | ((kTileM >> 4) << 24);
}

// Optional timestamps (clock64) of CTA 0..7 for profiling the pipeline: trace[cta][iteration][event]. Compiled in
// only with -DPDLLM_ENABLE_TRACE; the release kernel carries no trace code and ignores the pointer.
#ifdef PDLLM_ENABLE_TRACE
#define PDLLM_TRACE_ON (a.trace != nullptr)
#else
#define PDLLM_TRACE_ON false
#endif
constexpr int kTraceEvents = 16;
constexpr int kTraceIters = 64;
constexpr int kTraceCtas = 8;
__device__ __forceinline__ void trace_event(const Args& a, int it, int ev) {
  // slots 0-3: the first four CTAs of the grid; slots 4-7: the last four (they run in the last wave)
  const int slot = blockIdx.x < 4 ? static_cast<int>(blockIdx.x)
                                  : (blockIdx.x + 4 >= gridDim.x ? 4 + static_cast<int>(blockIdx.x + 4 - gridDim.x) : -1);
  if (slot >= 0 && it < kTraceIters && (threadIdx.x & 31) == 0 && (threadIdx.x == 0 || threadIdx.x == 128 || threadIdx.x >= 256)) {
    long long t = clock64();
    if (it == kTraceIters - 2) asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));  // row 62: wall-clock nanoseconds
    a.trace[(static_cast<int64_t>(slot) * kTraceIters + it) * kTraceEvents + ev] = t;
  }
}

struct TileInfo {
  bool is_ctx;
  int key0;    // first key of the tile: context position, or new-row index
  int nvalid;  // keys of the tile that exist (<= 128)
};

__device__ __forceinline__ TileInfo tile_info(int t, int n_ctx_tiles, int ctx_len, int new_end) {
  TileInfo ti;
  ti.is_ctx = t < n_ctx_tiles;
  if (ti.is_ctx) {
    ti.key0 = t * kTileN;
    ti.nvalid = min(kTileN, ctx_len - ti.key0);
  } else {
    ti.key0 = (t - n_ctx_tiles) * kTileN;
    ti.nvalid = min(kTileN, new_end - ti.key0);
  }
  return ti;
}

// Merge of the split-KV partials of one query-tile row: out[row] = sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s,
// splits added in index order whoever runs it. Partials were written by other CTAs: read them past L1. 32 columns of
// every split are in flight per thread before they are reduced.
__device__ __forceinline__ void merge_split_row(const float* __restrict__ part_o, const float* __restrict__ part_ml, int S, int is_bf16,
                                                int64_t unit0, int r, uint8_t* out_row) {
  float M = -INFINITY;
  for (int s = 0; s < S; ++s) {
    const float ms = __ldcg(&part_ml[((unit0 + s) * 2 + 0) * kTileM + r]);
    if (ms > -INFINITY) M = fmaxf(M, ms);
  }
  float wsum = 0.f;
  for (int s = 0; s < S; ++s) {
    const float ms = __ldcg(&part_ml[((unit0 + s) * 2 + 0) * kTileM + r]);
    const float ls = __ldcg(&part_ml[((unit0 + s) * 2 + 1) * kTileM + r]);
    if (ms > -INFINITY) wsum += exp2f(ms - M) * ls;
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
#pragma unroll 1
  for (int d0 = 0; d0 < kHeadDim; d0 += 32) {
    float acc[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) acc[j] = 0.f;
#pragma unroll 2
    for (int s = 0; s < S; ++s) {
      const float ms = __ldcg(&part_ml[((unit0 + s) * 2 + 0) * kTileM + r]);
      if (ms == -INFINITY) continue;   // a neutral partial has no O data behind it
      const float ws = exp2f(ms - M);
      const float* po = part_o + (unit0 + s) * kHeadDim * kTileM + static_cast<int64_t>(d0) * kTileM + r;
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __ldcg(po + j * kTileM);
#pragma unroll
      for (int j = 0; j < 32; ++j) acc[j] = fmaf(ws, v[j], acc[j]);
    }
    uint32_t packed[16];
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
      if (is_bf16) {
        __nv_bfloat162 h = __floats2bfloat162_rn(acc[j] * inv, acc[j + 1] * inv);
        packed[j >> 1] = *reinterpret_cast<uint32_t*>(&h);
      } else {
        __half2 h = __floats2half2_rn(acc[j] * inv, acc[j + 1] * inv);
        packed[j >> 1] = *reinterpret_cast<uint32_t*>(&h);
      }
    }
    uint4* dst = reinterpret_cast<uint4*>(out_row + d0 * 2);
#pragma unroll
    for (int j = 0; j < 4; ++j) dst[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
  }
}

// Called by every thread of a CTA once its partials are written and fenced. The CTA that arrives last for its
// (sequence, KV head, query-tile pair) merges all splits of both query tiles: no CTA ever waits for another.
__device__ __forceinline__ void finish_split(const Args& a, int seq, int kvh, int pair, int q_start, int tokA, int n_tokA, int tokB,
                                             int n_tokB) {
  __shared__ int is_last;
  const int64_t pair_id = (static_cast<int64_t>(seq) * a.num_kv_heads + kvh) * a.q_pairs + pair;
  if (threadIdx.x == 0) {
    is_last = (atomicAdd(&a.split_arrivals[pair_id], 1) == a.num_splits - 1) ? 1 : 0;
    if (is_last) a.split_arrivals[pair_id] = 0;   // every split has arrived: leave the counter ready for the next launch
  }
  __syncthreads();
  if (!is_last || threadIdx.x >= 2 * kTileM) return;
  __threadfence();
  const int x = threadIdx.x >> 7;
  const int r = threadIdx.x & (kTileM - 1);
  const int tok0 = x == 0 ? tokA : tokB;
  const int n_tok = x == 0 ? n_tokA : n_tokB;
  const int tok_local = r / a.group;
  if (tok_local >= n_tok) return;
  const int head_local = r - tok_local * a.group;
  const int64_t unit0 = ((static_cast<int64_t>(seq) * a.num_kv_heads + kvh) * a.q_tiles + 2 * pair + x - a.tile0) * a.num_splits;
  uint8_t* out_row = reinterpret_cast<uint8_t*>(a.out) +
                     ((static_cast<int64_t>(q_start + tok0 + tok_local)) * a.out_stride + static_cast<int64_t>(kvh * a.group + head_local) * kHeadDim) * 2;
  merge_split_row(a.part_o, a.part_ml, a.num_splits, a.is_bf16, unit0, r, out_row);
}

template <bool kBf16>
__global__ void __launch_bounds__(kThreads, 1)
attn_sm100_kernel(const __grid_constant__ CUtensorMap q_map, const __grid_constant__ CUtensorMap kn_map,
                  const __grid_constant__ CUtensorMap vn_map, const __grid_constant__ CUtensorMap kc_map,
                  const __grid_constant__ CUtensorMap vc_map, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kSmemBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kSmemBar + 256);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kSmemBar + 264);
  volatile int* tile_flags = reinterpret_cast<volatile int*>(smem + kSmemBar + 272);  // [4]: page of tile (it & 3) was unreadable

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  grid_dependency_wait();     // launched ahead of its predecessor's end: nothing global is touched before this
  grid_launch_dependents();

  // ---- decode the work unit: (sequence, KV head, pair of query tiles, KV split) ----
  // Unsplit units come first in launch order, then the split ones with the split as the slowest index: all first
  // splits, all second splits, ... With an uneven two-way split the first are the long CTAs, so the short second
  // splits fill in behind them and the last wave stays short.
  int u, split;
  if (static_cast<int>(blockIdx.x) < a.n_whole) {
    u = blockIdx.x; split = 0;
  } else {
    const int idx = blockIdx.x - a.n_whole, rest = a.base_ctas - a.n_whole;
    u = a.n_whole + idx % rest; split = idx / rest;
  }
  // CTAs that share this unit's key tiles (recomputed where it is needed rather than kept in a register)
#define PDLLM_NSPLIT (static_cast<int>(blockIdx.x) < a.n_whole ? 1 : a.num_splits)
  const int pair = u % a.q_pairs; u /= a.q_pairs;
  const int kvh = u % a.num_kv_heads;
  const int seq = u / a.num_kv_heads;

  const int q_start = a.cu_seqlens_q[seq];
  const int q_len = a.cu_seqlens_q[seq + 1] - q_start;
  int ctx_len = a.has_cache ? (a.seq_lens[seq] - q_len) : 0;
  if (ctx_len < 0) ctx_len = 0;
  const int G = a.group;
  // query tile X (0 = A, 1 = B) covers tokens [tok0[X], tok0[X] + n_tok[X])
  const int tokA = (2 * pair) * a.tpt, tokB = (2 * pair + 1) * a.tpt;
  const int n_tokA = min(a.tpt, q_len - tokA), n_tokB = min(a.tpt, q_len - tokB);
  const bool b_active = n_tokB > 0;
  const int n_q = b_active ? 2 : 1;

  // keys among the new rows that any row of this CTA may see (tile B holds the later rows)
  int new_end = q_len;
  if (n_tokA > 0) {
    const int last_m = b_active ? (tokB + n_tokB - 1) : (tokA + n_tokA - 1);
    if (a.mask_mode == PDLLM_MASK_CAUSAL) new_end = min(q_len, last_m + 1);
    else if (!a.bidirectional) new_end = min(q_len, (last_m / a.block_m + 1) * a.block_m);
  }
  const int n_ctx_tiles = (ctx_len + kTileN - 1) / kTileN;
  const int n_new_tiles = (new_end + kTileN - 1) / kTileN;
  const int total_tiles = n_ctx_tiles + n_new_tiles;
  int t_begin, t_end;
  if (a.first_permille > 0 && PDLLM_NSPLIT == 2) {   // two splits: [0, cut) and [cut, total)
    const int cut = min(total_tiles, (total_tiles * a.first_permille + 999) / 1000);
    t_begin = split == 0 ? 0 : cut;
    t_end = split == 0 ? cut : total_tiles;
  } else {
    const int nsplit = PDLLM_NSPLIT;
    const int per_split = (total_tiles + nsplit - 1) / nsplit;
    t_begin = split * per_split;
    t_end = min(total_tiles, t_begin + per_split);
  }
  const int n_iter = t_end - t_begin;
  // index of a query tile's split-KV partial
  const int64_t unit_base = ((static_cast<int64_t>(seq) * a.num_kv_heads + kvh) * a.q_tiles + 2 * pair - a.tile0) * a.num_splits + split;

  if (n_tokA <= 0) return;
  if (n_iter <= 0) {
    // Nothing to attend in this split: publish neutral partials so the merge ignores them.
    if (PDLLM_NSPLIT > 1 && threadIdx.x < 2 * kTileM && (threadIdx.x < kTileM || b_active)) {
      const int64_t unit = unit_base + (threadIdx.x >> 7) * a.num_splits;
      const int r = threadIdx.x & (kTileM - 1);
      a.part_ml[(unit * 2 + 0) * kTileM + r] = -INFINITY;
      a.part_ml[(unit * 2 + 1) * kTileM + r] = 0.f;
    }
    if (PDLLM_NSPLIT > 1 && a.fused_merge) {
      __threadfence();
      __syncthreads();
      finish_split(a, seq, kvh, pair, q_start, tokA, n_tokA, tokB, n_tokB);
    }
    return;
  }

  // ---- set-up: barriers, TMEM ----
  if (warp == kProducerWarp) {
    if (lane == 0) {
      for (int i = 0; i < kNumBars; ++i) {
        mbar_init(&bars[i], (i >= kPFull && i < kPFull + 4) ? 128u : (i >= kKFree ? static_cast<uint32_t>(n_q) : 1u));
      }
      abort_flag[0] = 0;
      fence_barrier_init();
    }
    __syncwarp();
    tmem_alloc(tmem_slot, kTmemCols);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const uint32_t idesc_qk = make_idesc(kBf16, false, kHalfN);    // S_Xb[128 x 64] = Q_X[128 x 128] K_b^T
  const uint32_t idesc_pv = make_idesc(kBf16, true, kHeadDim);   // O_X[128 x 128] += P_Xb[128 x 64] V_b

  if (warp == kProducerWarp) {
    // =========================== TMA producer ===========================
    // Key half-tiles h = 2*it + b stream through two rings of kRing slots (K and V). Slot h % kRing is free again
    // once both query tiles' MMAs on half-tile h - kRing are done (the K-free / V-free barriers).
    if (lane == 0) {
      const uint32_t q_bytes = 2u * 64u * 2u * static_cast<uint32_t>(G * a.tpt);
      mbar_expect_tx(&bars[kQFull], q_bytes * n_q);
      for (int x = 0; x < n_q; ++x) {
        const int tok0 = x == 0 ? tokA : tokB;
        tma_load_3d(&q_map, &bars[kQFull], smem + kSmemQ + x * kTileBytes, 0, kvh * G, q_start + tok0);
        tma_load_3d(&q_map, &bars[kQFull], smem + kSmemQ + x * kTileBytes + kHalfBytes, 64, kvh * G, q_start + tok0);
      }
      auto load_half = [&](bool is_v, int h) {
        const int it = h >> 1, b = h & 1;
        const int slot = h % kRing;
        const TileInfo ti = tile_info(t_begin + it, n_ctx_tiles, ctx_len, new_end);
        uint64_t* bar = &bars[(is_v ? kVFull : kKFull) + slot];
        uint8_t* dst = smem + (is_v ? kSmemV : kSmemK) + slot * kSlotBytes;
        mbar_expect_tx(bar, kSlotBytes);
        // one copy per slot: the tensor maps put the two 64-column halves of the head dimension in their outermost
        // box dimension, so the slot receives [half][64 keys][128 B]
        if (ti.is_ctx) {
          const int pidx = ti.key0 / a.page_size;
          const int off = ti.key0 - pidx * a.page_size + b * kHalfN;
          int page = (pidx < a.max_pages) ? a.block_table[seq * a.block_table_stride + pidx] : -1;
          const bool bad_page = page < 0 || page >= a.num_pages;
          if (bad_page) {
            report_status(a.status, PDLLM_S_BAD_PAGE);
            page = 0;  // keep the copy in bounds; the softmax warps hide the whole tile
          }
          if (!is_v && b == 0) tile_flags[it & 3] = bad_page ? 1 : 0;  // reaches the softmax warps through K-full → S-full
          tma_load_5d(is_v ? &vc_map : &kc_map, bar, dst, 0, off, 0, kvh, page);
        } else {
          if (!is_v && b == 0) tile_flags[it & 3] = 0;
          tma_load_4d(is_v ? &vn_map : &kn_map, bar, dst, 0, q_start + ti.key0 + b * kHalfN, 0, kvh);
        }
      };
      const int n_half = 2 * n_iter;
      for (int h = 0; h < n_half && h < kRing; ++h) load_half(false, h);
      for (int h = 0; h < n_half && h < kRing; ++h) load_half(true, h);
      bool ok = true;
      for (int h = 0; h + kRing < n_half && ok; ++h) {
        // a slot's "free" barrier completes once per use of the slot, and the slot cannot be used again before this
        // loop refills it, so the wait below is never more than one phase behind
        const int slot = h % kRing;
        const uint32_t use = (h / kRing) & 1;
        ok = mbar_wait<true>(&bars[kKFree + slot], use, abort_flag, a);   // every Q·K on half-tile h is done
        if (ok) load_half(false, h + kRing);
        if (ok) ok = mbar_wait<true>(&bars[kVFree + slot], use, abort_flag, a);  // every P·V on half-tile h is done
        if (ok) load_half(true, h + kRing);
      }
      // Every copy issued above is consumed by an MMA that the epilogue waits for, unless a wait gave up; then the
      // CTA is abandoning its result and only has to let copies in flight land: give them a bounded moment.
      if (!ok) {
        const long long t0 = clock64();
        while (clock64() - t0 < 200000) { }
      }
    }
    __syncwarp();
  } else if (warp >= kMmaWarp0) {
    // =========================== MMA issuers: one warp per chain (query tile x, key half b) ===========================
    // A single thread sustains only about one tcgen05.mma per ~110 cycles; four concurrent issuers keep the tensor
    // pipe fed. Each chain loops: P·V_xb(tile) once its softmax warps delivered P, then Q·K_xb of the next tile as
    // soon as that product released the S/P columns.
    const int chain = warp - kMmaWarp0;
    const int x = chain >> 1, b = chain & 1;
    if (x < n_q) {
    const uint32_t sq = smem_u32(smem + kSmemQ) + x * kTileBytes, sk = smem_u32(smem + kSmemK), sv = smem_u32(smem + kSmemV);
    const uint32_t tS = tmem_base + kColS + chain * kHalfN;   // S_xb, then P_xb in its first 32 columns
    const uint32_t tO = tmem_base + kColO + x * kHeadDim;
    auto issue_qk = [&](int slot) {   // S_xb = Q_x K_b^T
#pragma unroll
      for (int kk = 0; kk < kHeadDim / 16; ++kk) {
        const uint32_t qoff = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
        const uint32_t koff = slot * kSlotBytes + (kk >> 2) * (kSlotBytes / 2) + (kk & 3) * 32;
        umma_ss(tS, desc_kmajor_sw128(sq + qoff), desc_kmajor_sw128(sk + koff), idesc_qk, kk > 0 ? 1u : 0u);
      }
      umma_commit(&bars[kSFull + chain]);
      umma_commit(&bars[kKFree + slot]);
    };
    bool ok = mbar_wait<true>(&bars[kQFull], 0, abort_flag, a);
    if (ok) ok = mbar_wait<true>(&bars[kKFull + b], 0, abort_flag, a);  // half-tile b of tile 0 sits in slot b, first use
    if (ok) {
      tc_fence_after();
      if (lane == 0) issue_qk(b);
      __syncwarp();
    }
    for (int it = 0; it < n_iter && ok; ++it) {
      const uint32_t ph = it & 1;
      const TileInfo ti = tile_info(t_begin + it, n_ctx_tiles, ctx_len, new_end);
      const int h = 2 * it + b;
      const int slot = h % kRing;
      ok = mbar_wait<true>(&bars[kVFull + slot], (h / kRing) & 1, abort_flag, a);
      if (!ok) break;
      if (ti.nvalid < (b + 1) * kHalfN) {
        // Rows of V_b past the last valid key may hold anything (stale page contents, another sequence's
        // rows); P is 0 there but 0 * NaN is NaN, so clear them before the MMA reads the half tile. Both query
        // tiles' issuers do this for the slot they share: the writes are identical zeros.
        const int first = max(ti.nvalid, b * kHalfN) - b * kHalfN;  // first row to clear inside the slot
        const int n_rows = kHalfN - first;
        for (int i = lane; i < n_rows * 16; i += 32) {
          const int r = first + (i >> 4);
          const int c = i & 15;
          uint4* dst = reinterpret_cast<uint4*>(smem + kSmemV + slot * kSlotBytes + (c >> 3) * (kSlotBytes / 2) + r * 128 + (c & 7) * 16);
          *dst = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async();
        __syncwarp();
      }
      ok = mbar_wait<true>(&bars[kPFull + chain], ph, abort_flag, a);
      // O_x is accumulated by both chains of query tile x, from two threads: keep their products strictly
      // alternating (x,0)(x,1)(x,0)... by waiting for the sibling's previous product. The softmax warps deliver P in
      // that order anyway, so this wait is normally already satisfied.
      if (ok && b == 1) ok = mbar_wait<true>(&bars[kPvDone + chain - 1], ph, abort_flag, a);
      if (ok && b == 0 && it > 0) ok = mbar_wait<true>(&bars[kPvDone + chain + 1], ph ^ 1, abort_flag, a);
      if (!ok) break;
      tc_fence_after();
      if (PDLLM_TRACE_ON) trace_event(a, it, 4 + chain);
      if (lane == 0) {
#pragma unroll
        for (int kk = 0; kk < kHalfN / 16; ++kk) {
          umma_ts(tO, tS + kk * 8, desc_mnmajor_sw128(sv + slot * kSlotBytes + kk * 2048, kSlotBytes / 2), idesc_pv,
                  (it > 0 || b > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&bars[kPvDone + chain]);
        umma_commit(&bars[kVFree + slot]);
      }
      __syncwarp();
      if (it + 1 < n_iter) {
        const int hn = h + 2;
        const int nslot = hn % kRing;
        ok = mbar_wait<true>(&bars[kKFull + nslot], (hn / kRing) & 1, abort_flag, a);
        if (ok) ok = mbar_wait<true>(&bars[kPvDone + chain], ph, abort_flag, a);  // S_xb / P_xb columns are free again
        if (!ok) break;
        tc_fence_after();
        if (PDLLM_TRACE_ON) trace_event(a, it, 12 + chain);
        if (lane == 0) issue_qk(nslot);
        __syncwarp();
      }
    }
    }  // x < n_q
  } else {
    // =========================== softmax + epilogue (warps 0-3: query tile A, warps 4-7: query tile B) ===========
    const int x = warp >> 2;
    if (x < n_q) {
    const int r = threadIdx.x & (kTileM - 1);   // tile row == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem_base + lane_base + kColS + x * 2 * kHalfN;
    const uint32_t tO = tmem_base + lane_base + kColO + x * kHeadDim;
    const int tok0 = x == 0 ? tokA : tokB;
    const int n_tok = x == 0 ? n_tokA : n_tokB;
    const int tok_local = r / G;               // token of this row inside the tile
    const int head_local = r - tok_local * G;
    const bool row_valid = tok_local < n_tok;
    const int m = tok0 + tok_local;            // sequence-local new-row index
    const int64_t unit = unit_base + x * a.num_splits;
    // last visible new key (exclusive) for this row
    int row_new_end = q_len;
    if (a.mask_mode == PDLLM_MASK_CAUSAL) row_new_end = min(q_len, m + 1);
    else if (!a.bidirectional) row_new_end = min(q_len, (m / a.block_m + 1) * a.block_m);
    const bool dense_mask = (a.mask != nullptr) && (a.mask_mode == PDLLM_MASK_BLOCK);

    float m_ref = -INFINITY;  // running reference maximum, log2 domain
    float l_run = 0.f;
    bool ok = true;
    uint32_t s[kHalfN];       // one row of one S buffer; the epilogue reuses it for O
    if (PDLLM_TRACE_ON) { trace_event(a, kTraceIters - 1, 0); trace_event(a, kTraceIters - 2, 0); }
    constexpr uint32_t kNegInf = 0xff800000u;

    for (int it = 0; it < n_iter && ok; ++it) {
      const uint32_t ph = it & 1;
      const TileInfo ti = tile_info(t_begin + it, n_ctx_tiles, ctx_len, new_end);
      int cmax_tile = ti.nvalid;  // columns [0, cmax_tile) of the 128-key tile are visible to this row
      if (!ti.is_ctx) cmax_tile = min(cmax_tile, row_new_end - ti.key0);
      const bool use_dense = dense_mask && !ti.is_ctx && row_valid;
      const uint8_t* mrow = use_dense ? a.mask + static_cast<int64_t>(m) * a.mask_stride_m + static_cast<int64_t>(ti.key0) * a.mask_stride_n : nullptr;

#pragma unroll
      for (int b = 0; b < 2; ++b) {
        const uint32_t tSb = tS + b * kHalfN;
        ok = mbar_wait(&bars[kSFull + x * 2 + b], ph, abort_flag, a);
        if (!ok) break;
        tc_fence_after();
        if (PDLLM_TRACE_ON) trace_event(a, it, x * 2 + b);

        tmem_ld32(tSb, s);
        tmem_ld32(tSb + 32, s + 32);
        tc_wait_ld();
        int cmax = cmax_tile - b * kHalfN;
        if (tile_flags[it & 3]) cmax = 0;  // the producer could not read this tile's page: hide all of it
        if (cmax < kHalfN || use_dense) {
#pragma unroll
          for (int j = 0; j < kHalfN; ++j) {
            bool vis = j < cmax;
            if (vis && use_dense) vis = mrow[(b * kHalfN + j) * a.mask_stride_n] != 0;
            if (!vis) s[j] = kNegInf;
          }
        }

        // row maximum of this half, four independent chains
        float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
        for (int j = 0; j < kHalfN; j += 4) {
          mx0 = fmaxf(mx0, __uint_as_float(s[j]));
          mx1 = fmaxf(mx1, __uint_as_float(s[j + 1]));
          mx2 = fmaxf(mx2, __uint_as_float(s[j + 2]));
          mx3 = fmaxf(mx3, __uint_as_float(s[j + 3]));
        }
        const float m_half = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * a.scale_log2;  // scale > 0: max commutes

        // lazy rescale: only when the maximum grew by more than 2^8 (the very first half just sets the reference)
        if (it == 0 && b == 0) {
          m_ref = m_half;
        } else {
          const bool grow = m_half > m_ref + kRescaleThreshold;
          if (__any_sync(0xffffffffu, grow)) {
            // O must hold every product issued so far: the previous half's P·V may still be in flight
            const int pb = b ^ 1;
            const uint32_t pph = (b == 1) ? ph : (ph ^ 1);
            ok = mbar_wait(&bars[kPvDone + x * 2 + pb], pph, abort_flag, a);
            if (!ok) break;
            tc_fence_after();
            const float m_new = grow ? m_half : m_ref;
            const float alpha = grow ? ex2(m_ref - m_new) : 1.f;  // m_ref = -inf gives 0
            l_run *= alpha;
            uint32_t o[16];
#pragma unroll 1
            for (int c = 0; c < kHeadDim / 16; ++c) {
              tmem_ld16(tO + c * 16, o);
              tc_wait_ld();
#pragma unroll
              for (int j = 0; j < 16; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * alpha);
              tmem_st16(tO + c * 16, o);
            }
            tc_wait_st();
            m_ref = m_new;
          }
        }
        const float m_use = (m_ref == -INFINITY) ? 0.f : m_ref;

        // P_b = exp2(S_b*scale - m_ref) → bf16/fp16 pairs over the first 32 columns of S_b
        float l0 = 0.f, l1 = 0.f, l2 = 0.f, l3 = 0.f;
        uint32_t packed[kHalfN / 2];
#pragma unroll
        for (int j = 0; j < kHalfN; j += 4) {
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
        tmem_st32(tSb, packed);
        l_run += (l0 + l1) + (l2 + l3);
        tc_wait_st();
        tc_fence_before();
        mbar_arrive(&bars[kPFull + x * 2 + b]);
        if (PDLLM_TRACE_ON) trace_event(a, it, 8 + x * 2 + b);
      }
    }

    // ---- epilogue ----
    if (PDLLM_TRACE_ON) trace_event(a, kTraceIters - 1, 1);
    if (ok) ok = mbar_wait(&bars[kPvDone + x * 2 + 1], (n_iter - 1) & 1, abort_flag, a);  // in-order MMAs: the last P·V done implies all done
    if (PDLLM_TRACE_ON) trace_event(a, kTraceIters - 1, 2);
    if (ok) {
      tc_fence_after();
      if (PDLLM_NSPLIT == 1) {
        const float inv = (l_run > 0.f) ? 1.f / l_run : 0.f;
        uint8_t* out_row = reinterpret_cast<uint8_t*>(a.out) +
                           ((static_cast<int64_t>(q_start + m)) * a.out_stride + static_cast<int64_t>(kvh * G + head_local) * kHeadDim) * 2;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          tmem_ld32(tO + c * 32, s);
          tc_wait_ld();
          if (row_valid) {
            uint32_t packed[16];
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              const float o0 = __uint_as_float(s[j]) * inv, o1 = __uint_as_float(s[j + 1]) * inv;
              if (kBf16) {
                __nv_bfloat162 h = __floats2bfloat162_rn(o0, o1);
                packed[j >> 1] = *reinterpret_cast<uint32_t*>(&h);
              } else {
                __half2 h = __floats2half2_rn(o0, o1);
                packed[j >> 1] = *reinterpret_cast<uint32_t*>(&h);
              }
            }
            uint4* dst = reinterpret_cast<uint4*>(out_row + c * 64);
#pragma unroll
            for (int j = 0; j < 4; ++j) dst[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
          }
        }
      } else {
        float* po = a.part_o + unit * kHeadDim * kTileM;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          tmem_ld32(tO + c * 32, s);
          tc_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) po[static_cast<int64_t>(c * 32 + j) * kTileM + r] = __uint_as_float(s[j]);
        }
        a.part_ml[(unit * 2 + 0) * kTileM + r] = m_ref;
        a.part_ml[(unit * 2 + 1) * kTileM + r] = l_run;
      }
    }
    if (PDLLM_TRACE_ON) { trace_event(a, kTraceIters - 1, 3); trace_event(a, kTraceIters - 2, 1); }
    }  // x < n_q
  }

  // ---- teardown ----
  tc_fence_before();
  if (PDLLM_NSPLIT > 1 && a.fused_merge) __threadfence();   // this CTA's partials are visible before it counts itself in
  __syncthreads();
  if (warp == kProducerWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if (PDLLM_NSPLIT > 1 && a.fused_merge) finish_split(a, seq, kvh, pair, q_start, tokA, n_tokA, tokB, n_tokB);
#undef PDLLM_NSPLIT
}

// Stand-alone merge for shapes with few (sequence, KV head, tile pair) units and many splits (a single block of
// decode rows): there the fused merge would pull S partial tiles through ONE SM per unit, while this grid spreads the
// same reads over (query tiles x 8 column slabs) CTAs. Thread r owns tile row r and 16 columns; 64 loads in flight.
constexpr int kCombineCols = 16;
__global__ void __launch_bounds__(kTileM) attn_combine_kernel(const Args a) {
  const int64_t tile = blockIdx.x / (kHeadDim / kCombineCols);  // (seq, kvh, qt)
  const int d0 = static_cast<int>(blockIdx.x % (kHeadDim / kCombineCols)) * kCombineCols;
  int u = static_cast<int>(tile);
  const int qt = u % a.q_tiles; u /= a.q_tiles;
  const int kvh = u % a.num_kv_heads;
  const int seq = u / a.num_kv_heads;
  const int q_start = a.cu_seqlens_q[seq];
  const int q_len = a.cu_seqlens_q[seq + 1] - q_start;
  const int tok0 = qt * a.tpt;
  const int n_tok = min(a.tpt, q_len - tok0);
  const int r = threadIdx.x;
  const int tok_local = r / a.group;
  if (n_tok <= 0 || tok_local >= n_tok) return;
  const int head_local = r - tok_local * a.group;
  const int64_t unit0 = tile * a.num_splits;
  const int S = a.num_splits;
  float M = -INFINITY;
  for (int s = 0; s < S; ++s) M = fmaxf(M, a.part_ml[((unit0 + s) * 2 + 0) * kTileM + r]);
  float wsum = 0.f;
  for (int s = 0; s < S; ++s) {
    const float ms = a.part_ml[((unit0 + s) * 2 + 0) * kTileM + r];
    if (ms > -INFINITY) wsum += exp2f(ms - M) * a.part_ml[((unit0 + s) * 2 + 1) * kTileM + r];
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  float acc[kCombineCols];
#pragma unroll
  for (int j = 0; j < kCombineCols; ++j) acc[j] = 0.f;
#pragma unroll 4
  for (int s = 0; s < S; ++s) {
    const float ms = a.part_ml[((unit0 + s) * 2 + 0) * kTileM + r];
    const float ws = ms == -INFINITY ? 0.f : exp2f(ms - M);   // a neutral partial has no O data behind it
    const float* po = a.part_o + (unit0 + s) * kHeadDim * kTileM + static_cast<int64_t>(d0) * kTileM + r;
    float v[kCombineCols];
#pragma unroll
    for (int j = 0; j < kCombineCols; ++j) v[j] = ws != 0.f ? po[j * kTileM] : 0.f;
#pragma unroll
    for (int j = 0; j < kCombineCols; ++j) acc[j] = fmaf(ws, v[j], acc[j]);
  }
  uint32_t packed[kCombineCols / 2];
#pragma unroll
  for (int j = 0; j < kCombineCols; j += 2) {
    if (a.is_bf16) {
      __nv_bfloat162 h = __floats2bfloat162_rn(acc[j] * inv, acc[j + 1] * inv);
      packed[j >> 1] = *reinterpret_cast<uint32_t*>(&h);
    } else {
      __half2 h = __floats2half2_rn(acc[j] * inv, acc[j + 1] * inv);
      packed[j >> 1] = *reinterpret_cast<uint32_t*>(&h);
    }
  }
  uint8_t* out_row = reinterpret_cast<uint8_t*>(a.out) +
                     ((static_cast<int64_t>(q_start + tok0 + tok_local)) * a.out_stride + static_cast<int64_t>(kvh * a.group + head_local) * kHeadDim) * 2;
  uint4* dst = reinterpret_cast<uint4*>(out_row + d0 * 2);
  dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
}

// ---- host side: tensor maps, split choice, launch ---------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                                  const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qres;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qres) == cudaSuccess &&
        qres == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  });
  return fn;
}

// rank-3 or rank-4 map over 2-byte elements, 128-byte swizzle, zero fill outside the tensor
inline int encode_map(CUtensorMap* map, bool bf16, const void* base, int rank, const uint64_t* dims,
                      const uint64_t* strides_bytes /* rank-1 entries */, const uint32_t* box) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(PDLLM_E_DRIVER, "cuTensorMapEncodeTiled entry point not available");
  cuuint64_t gdim[5]; cuuint64_t gstr[4]; cuuint32_t bdim[5]; cuuint32_t estr[5];
  for (int i = 0; i < rank; ++i) { gdim[i] = dims[i]; bdim[i] = box[i]; estr[i] = 1; }
  for (int i = 0; i < rank - 1; ++i) gstr[i] = strides_bytes[i];
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, rank,
                  const_cast<void*>(base), gdim, gstr, bdim, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PDLLM_E_DRIVER, "cuTensorMapEncodeTiled failed with CUresult %d", static_cast<int>(r));
  return 0;
}

inline bool supported(const pdllm_attn_params* p, const char** why) {
  const char* w = nullptr;
  if (p->dtype != PDLLM_BF16 && p->dtype != PDLLM_F16) w = "dtype must be bf16 or fp16";
  else if (p->head_dim != kHeadDim) w = "head_dim must be 128";
  else if (p->num_q_heads % p->num_kv_heads != 0) w = "query heads must be a multiple of KV heads";
  else if (p->num_q_heads / p->num_kv_heads > kTileM) w = "GQA group larger than 128";
  else if (p->kv_layout == PDLLM_KV_DISTINCT) w = "distinct cache layout runs on the SIMT kernel";
  else if (p->kv_layout == PDLLM_KV_UNIFIED && (p->page_size % kTileN != 0)) w = "page_size must be a multiple of 128";
  else if (p->kv_layout == PDLLM_KV_UNIFIED && p->page_size > 256 * kTileN) w = "page_size too large";
  else if ((reinterpret_cast<uintptr_t>(p->q) | reinterpret_cast<uintptr_t>(p->k_new) | reinterpret_cast<uintptr_t>(p->v_new) |
            reinterpret_cast<uintptr_t>(p->out) | reinterpret_cast<uintptr_t>(p->k_cache) | reinterpret_cast<uintptr_t>(p->v_cache)) & 15) w = "pointers must be 16-byte aligned";
  else if ((p->q_stride | p->k_stride | p->v_stride | p->out_stride) % 8 != 0) w = "row strides must be multiples of 8 elements";
  else if (p->total_q >= (1ll << 31) || p->num_pages >= (1ll << 31)) w = "extent exceeds the tensor-map coordinate range";
  if (why) *why = w;
  return w == nullptr;
}

struct Plan {
  int group, tpt, q_tiles, q_pairs, num_splits;
  int first_permille;  // see Args
  int fused_merge;     // see Args
  int64_t tiles;  // query tiles
  int64_t units;  // (sequence, KV head, query-tile pair) units
  int64_t n_whole;  // units that run unsplit, see Args
  int64_t tile0;    // first query tile that has split-KV partials, see Args
  int64_t ctas;   // CTAs launched: n_whole + (units - n_whole) x splits
};

inline Plan make_plan(const pdllm_attn_params* p) {
  Plan pl;
  pl.group = p->num_q_heads / p->num_kv_heads;
  pl.tpt = kTileM / pl.group;
  pl.q_tiles = (p->max_query_len + pl.tpt - 1) / pl.tpt;
  if (pl.q_tiles < 1) pl.q_tiles = 1;
  pl.q_pairs = (pl.q_tiles + 1) / 2;
  pl.tiles = static_cast<int64_t>(p->num_seqs) * p->num_kv_heads * pl.q_tiles;
  const int64_t base_ctas = static_cast<int64_t>(p->num_seqs) * p->num_kv_heads * pl.q_pairs;
  int max_key_tiles = (p->max_seq_len + kTileN - 1) / kTileN + 1;
  int splits = p->num_splits;
  pl.first_permille = 0;
  const int64_t sms = sm_count();
  if (splits <= 0 && base_ctas < sms && 2 * base_ctas > sms && max_key_tiles >= 6) {
    // More units than half the SMs but fewer than all of them: an even split either leaves SMs idle (1 split) or
    // runs two full waves (3 splits). Cut every unit in two UNEVEN parts instead: the long parts occupy base_ctas SMs
    // for the whole kernel, the short parts run k at a time on each of the other SMs, and the cut makes both kinds
    // of SM finish together: long = ovh + B t, short = k (ovh + S t), B + S = T, with the per-CTA overhead ovh
    // (prologue, epilogue, its share of the merge) worth about 4.5 key-tile times t: the cut that was fastest on the
    // op-level shape (33 key tiles, 96 units, 148 SMs) is 24 + 9.
    const int64_t rest = sms - base_ctas;
    const int64_t k = (base_ctas + rest - 1) / rest;
    const double T = max_key_tiles - 1, ovh = 4.5;
    double S = (T - (k - 1) * ovh) / (k + 1);
    if (S >= 2.0) {
      splits = 2;
      pl.first_permille = static_cast<int>(1000.0 * (T - S) / T + 0.5);
      if (pl.first_permille < 500) pl.first_permille = 500;
      if (pl.first_permille > 950) pl.first_permille = 950;
    }
  }
  pl.fused_merge = 1;
  if (2 * base_ctas <= sms) {
    // Few units (the decode shape: one block of rows per request): everything fits in one wave, and the merge of S
    // partial tiles per unit is better spread over a grid of its own than pulled through the one SM that finishes
    // last. In key-tile times: cost(S) = ovh + ceil(T / S) + launch + merge * S, ovh ~ 2.3, launch ~ 1, merge ~ 0.25 (a sweep
    // at 32 rows x 4161 keys is flat between 8 and 16 splits, 28 us, and rises on both sides).
    pl.fused_merge = 0;
    if (splits <= 0) {
      const int T = max_key_tiles - 1;
      int64_t s_max = sms / base_ctas;
      if (s_max > 32) s_max = 32;
      if (s_max > T) s_max = T > 0 ? T : 1;
      double best = 2.3 + T;
      splits = 1;
      for (int s = 2; s <= s_max; ++s) {
        const double cost = 2.3 + (T + s - 1) / s + 1.0 + 0.25 * s;
        if (cost < best - 1e-9) { best = cost; splits = s; }
      }
    }
  }
  pl.n_whole = 0;
  if (splits <= 0) {
    // At least one unit per SM. Whole waves of unsplit units first (no partials, no merge), then the remaining units
    // cut into splits that fill the last wave(s), so that the tail of the kernel is a fraction of a unit long. In
    // key-tile times a wave costs its key tiles plus a per-CTA overhead of about 1 (unsplit) or 4 (split: partials
    // and merge): 16 x 32 units of 65 key tiles on 148 SMs ran 501 / 518 / 569 us with 1 / 2 / 3 even splits.
    const int64_t slots = sm_count();
    int cap = max_key_tiles / 4; if (cap < 1) cap = 1; if (cap > 8) cap = 8;   // a split keeps at least four key tiles
    const int T = max_key_tiles - 1 > 0 ? max_key_tiles - 1 : 1;
    double best = -1.0; splits = 1;
    for (int64_t w = base_ctas / slots; w >= 0; --w) {
      const int64_t rest = base_ctas - w * slots;
      for (int s = 1; s <= cap; ++s) {
        if (rest == 0 && s > 1) break;
        const int64_t waves = (rest * s + slots - 1) / slots;
        const double cost = static_cast<double>(w) * (1.0 + T) + static_cast<double>(waves) * ((s > 1 ? 4.0 : 1.0) + (T + s - 1) / s);
        if (best < 0.0 || cost < best * 0.97) { best = cost; splits = s; pl.n_whole = s > 1 ? w * slots : 0; }
      }
    }
  }
  if (splits > 32) splits = 32;
  if (splits > max_key_tiles) splits = max_key_tiles;
  if (splits < 1) splits = 1;
  if (splits == 1) pl.n_whole = 0;
  pl.num_splits = splits;
  pl.units = base_ctas;
  pl.tile0 = (pl.n_whole / pl.q_pairs) * pl.q_tiles + 2 * (pl.n_whole % pl.q_pairs);
  pl.ctas = pl.n_whole + (base_ctas - pl.n_whole) * splits;
  return pl;
}

// The arrival counters sit at the start of the workspace in a header of fixed size, so that a workspace that was
// zero-filled once keeps zeroed counters whatever shapes it serves (the kernel returns each counter to zero).
constexpr int64_t kCounterHeaderBytes = 64 * 1024;
inline int64_t counter_bytes(int64_t pairs) { return pairs * 4 <= kCounterHeaderBytes ? kCounterHeaderBytes : ((pairs * 4 + 255) / 256) * 256; }

inline int64_t workspace_bytes(const pdllm_attn_params* p) {
  Plan pl = make_plan(p);
  if (pl.num_splits <= 1) return 0;
  const int64_t pairs = static_cast<int64_t>(p->num_seqs) * p->num_kv_heads * pl.q_pairs;
  return counter_bytes(pairs) + (pl.tiles - pl.tile0) * pl.num_splits * (static_cast<int64_t>(kHeadDim) * kTileM + 2 * kTileM) * 4;
}

inline int launch(const pdllm_attn_params* p, cudaStream_t stream) {
  const char* why = nullptr;
  if (!supported(p, &why)) return fail(PDLLM_E_UNSUPPORTED, "tcgen05 attention: %s", why);
  if (p->total_q == 0 || p->num_seqs == 0) return 0;
  const Plan pl = make_plan(p);
  const bool bf16 = p->dtype == PDLLM_BF16;
  const bool has_cache = p->kv_layout == PDLLM_KV_UNIFIED && p->k_cache != nullptr && p->num_pages > 0;

  if (pl.num_splits > 1) {
    const int64_t need = workspace_bytes(p);
    if (p->workspace == nullptr || p->workspace_bytes < need) {
      return fail(PDLLM_E_WORKSPACE, "attention needs %lld workspace bytes for %d KV splits, got %lld",
                  static_cast<long long>(need), pl.num_splits, static_cast<long long>(p->workspace_bytes));
    }
  }

  CUtensorMap q_map, kn_map, vn_map, kc_map, vc_map;
  int rc;
  {
    uint64_t dims[3] = {static_cast<uint64_t>(kHeadDim), static_cast<uint64_t>(p->num_q_heads), static_cast<uint64_t>(p->total_q)};
    uint64_t str[2] = {static_cast<uint64_t>(kHeadDim) * 2, static_cast<uint64_t>(p->q_stride) * 2};
    uint32_t box[3] = {64, static_cast<uint32_t>(pl.group), static_cast<uint32_t>(pl.tpt)};
    if ((rc = encode_map(&q_map, bf16, p->q, 3, dims, str, box)) != 0) return rc;
  }
  {
    // new K/V rows [T, Hkv, D] seen as (64 cols, T rows, 2 column halves, Hkv): one box = [2][64 rows][64 cols]
    uint64_t dims[4] = {64, static_cast<uint64_t>(p->total_q), 2, static_cast<uint64_t>(p->num_kv_heads)};
    uint32_t box[4] = {64, kHalfN, 2, 1};
    uint64_t strk[3] = {static_cast<uint64_t>(p->k_stride) * 2, 128, static_cast<uint64_t>(kHeadDim) * 2};
    uint64_t strv[3] = {static_cast<uint64_t>(p->v_stride) * 2, 128, static_cast<uint64_t>(kHeadDim) * 2};
    if ((rc = encode_map(&kn_map, bf16, p->k_new, 4, dims, strk, box)) != 0) return rc;
    if ((rc = encode_map(&vn_map, bf16, p->v_new, 4, dims, strv, box)) != 0) return rc;
  }
  if (has_cache) {
    // pool [pages, page_size, Hkv, D] seen as (64 cols, page_size rows, 2 column halves, Hkv, pages)
    const uint64_t row = static_cast<uint64_t>(kHeadDim) * 2 * p->num_kv_heads;
    uint64_t dims[5] = {64, static_cast<uint64_t>(p->page_size), 2, static_cast<uint64_t>(p->num_kv_heads), static_cast<uint64_t>(p->num_pages)};
    uint64_t str[4] = {row, 128, static_cast<uint64_t>(kHeadDim) * 2, row * p->page_size};
    uint32_t box[5] = {64, kHalfN, 2, 1, 1};
    if ((rc = encode_map(&kc_map, bf16, p->k_cache, 5, dims, str, box)) != 0) return rc;
    if ((rc = encode_map(&vc_map, bf16, p->v_cache, 5, dims, str, box)) != 0) return rc;
  } else {
    kc_map = kn_map; vc_map = vn_map;  // never dereferenced: no context tiles exist
  }

  Args a;
  a.out = p->out; a.block_table = p->block_table; a.cu_seqlens_q = p->cu_seqlens_q; a.seq_lens = p->seq_lens;
  a.mask = p->mask; a.status = p->status;
  a.trace = reinterpret_cast<long long*>(p->trace);
  const int64_t pairs = static_cast<int64_t>(p->num_seqs) * p->num_kv_heads * pl.q_pairs;
  a.split_arrivals = reinterpret_cast<int*>(p->workspace);
  a.part_o = p->workspace ? reinterpret_cast<float*>(static_cast<char*>(p->workspace) + counter_bytes(pairs)) : nullptr;
  a.part_ml = a.part_o ? a.part_o + (pl.tiles - pl.tile0) * pl.num_splits * static_cast<int64_t>(kHeadDim) * kTileM : nullptr;
  if (pl.num_splits > 1 && pl.fused_merge && !(p->workspace_zeroed && pairs * 4 <= kCounterHeaderBytes)) {
    // The kernel leaves every counter at zero again, so a caller that zero-filled its workspace once (and again after
    // any launch that reported a wait time-out) can say so and save this memset node on every call.
    cudaError_t e = cudaMemsetAsync(a.split_arrivals, 0, static_cast<size_t>(pairs) * 4, stream);
    if (e != cudaSuccess) return fail(static_cast<int>(e), "cudaMemsetAsync(split counters): %s", cudaGetErrorString(e));
  }
  a.out_stride = p->out_stride; a.block_table_stride = p->block_table_stride;
  a.mask_stride_m = p->mask_stride_m; a.mask_stride_n = p->mask_stride_n; a.num_pages = has_cache ? p->num_pages : 0;
  a.num_seqs = p->num_seqs; a.max_pages = p->max_pages; a.num_q_heads = p->num_q_heads; a.num_kv_heads = p->num_kv_heads;
  a.group = pl.group; a.tpt = pl.tpt; a.q_tiles = pl.q_tiles; a.q_pairs = pl.q_pairs; a.num_splits = pl.num_splits;
  a.first_permille = pl.num_splits == 2 ? pl.first_permille : 0;
  a.base_ctas = static_cast<int>(pl.units); a.n_whole = static_cast<int>(pl.n_whole); a.tile0 = static_cast<int>(pl.tile0);
  a.fused_merge = pl.fused_merge;
  a.page_size = p->page_size > 0 ? p->page_size : kTileN; a.has_cache = has_cache ? 1 : 0;
  a.mask_mode = p->mask_mode; a.bidirectional = p->bidirectional;
  a.block_m = 2 * (p->diffusion_blk > 0 ? p->diffusion_blk : 32);
  a.is_bf16 = bf16 ? 1 : 0;
  a.scale_log2 = p->sm_scale * 1.4426950408889634f;

  {
    // the opt-in shared-memory size is a per-device function attribute
    static std::mutex mu;
    static bool done[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 0 || dev >= 64 || !done[dev]) {
      cudaError_t e = cudaFuncSetAttribute(attn_sm100_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
      if (e == cudaSuccess) e = cudaFuncSetAttribute(attn_sm100_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
      if (e != cudaSuccess) return fail(static_cast<int>(e), "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      if (dev >= 0 && dev < 64) done[dev] = true;
    }
  }

  if (bf16) (void)launch_dependent(attn_sm100_kernel<true>, dim3(static_cast<unsigned>(pl.ctas)), dim3(kThreads), kSmemBytes, stream, q_map, kn_map, vn_map, kc_map, vc_map, a);
  else (void)launch_dependent(attn_sm100_kernel<false>, dim3(static_cast<unsigned>(pl.ctas)), dim3(kThreads), kSmemBytes, stream, q_map, kn_map, vn_map, kc_map, vc_map, a);
  if ((rc = check_launch("attn_sm100_kernel")) != 0) return rc;
  if (pl.num_splits > 1 && !pl.fused_merge) {
    attn_combine_kernel<<<static_cast<unsigned>(pl.tiles * (kHeadDim / kCombineCols)), kTileM, 0, stream>>>(a);
    if ((rc = check_launch("attn_combine_kernel")) != 0) return rc;
  }
  return 0;
}

}  // namespace tc
}  // namespace pdllm
