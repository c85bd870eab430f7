// Linear layers on the 5th-generation tensor cores (sm_100a): out[M, N] = x[M, K] · W[N, K]^T (+ bias) with an optional
// fused SiLU(gate)·up epilogue, for the QKV / O / gate-up / down projections and the LM head of the Dream / LLaDA block.
// bf16 or fp16 operands, fp32 accumulation in TMEM, operands staged by TMA (128-byte swizzle) through a ring of
// shared-memory stages, one thread issuing tcgen05.mma, eight warps draining the accumulator.
//
// Both operands are K-major ([rows, K] row-major), so either can be the 128-row "A" side of the instruction:
//   * few rows (M <= 128: one block of decode rows, a draft, a commit): the WEIGHTS are A. A CTA streams 128 weight rows
//     x K through shared memory once, the activations are the narrow B side (16..128 columns), the accumulator is
//     out^T [128 features x M tokens]. The step is bound by reading the weights from HBM, so the (feature tile, k-block)
//     units are dealt to the CTAs stream-K style: every CTA of the grid (one per SM) gets the same number of 16 KB weight
//     blocks to stream, whatever N and K are; a feature tile that ends up spread over several CTAs is summed by the CTA
//     that finishes it last, in CTA order, through fp32 partials in the workspace (an arrival counter per tile; no CTA
//     ever waits for another). A product with few feature tiles (QKV, O, down of a 7B model) instead gives every tile to a
//     thread-block cluster whose CTAs split its k-blocks and send one another their shares with asynchronous copies between
//     shared memories.
//   * many rows (prefill, scoring): the ACTIVATIONS are A: tiles of 128 tokens x 256 (or 128) features, all of K per tile,
//     tiles dealt round-robin with the token tiles of one weight tile adjacent so that concurrent CTAs share it in L2; from
//     512 rows, tiles of 256 tokens x 256 features worked by PAIRS of CTAs: one tcgen05.mma over two SMs (cta_group::2), each
//     CTA staging its 128 token rows and half of the weight rows.
// The accumulator is double-buffered in TMEM: while the epilogue warps drain tile i, the tensor core works on tile i+1.
// Every mbarrier wait is bounded; on expiry the CTA raises PDLLM_S_WAIT_TIMEOUT, stops issuing and frees its TMEM.
#pragma once

#include <type_traits>

#include "attn_sm100.cuh"

namespace pdllm {
namespace gemm {

using tc::mbar_init; using tc::mbar_expect_tx; using tc::mbar_arrive; using tc::mbar_wait; using tc::smem_u32;
using tc::fence_barrier_init; using tc::tc_fence_before; using tc::tc_fence_after; using tc::tc_wait_ld;
using tc::umma_ss; using tc::umma_commit; using tc::desc_kmajor_sw128; using tc::make_idesc;

constexpr int kRowsA = 128;            // rows of the A tile = TMEM lanes
constexpr int kBlockK = 64;            // elements of K per stage: one 128-byte swizzle row
constexpr int kThreads = 320;          // warp 0: TMA producer, warp 1: MMA issuer + TMEM owner, warps 2-9: epilogue
constexpr int kEpiWarp0 = 2;
constexpr int kEpiThreads = 256;       // two warps per TMEM lane quarter: they take alternate 16-column chunks of the accumulator
constexpr int kSmemBudget = 200 * 1024;
constexpr int kSmemLimit = 224 * 1024;  // ring + receive buffer + barriers stay under the 227 KB a CTA may have
// Few rows: room for the shares of an accumulator that the CTAs of a cluster send one another (fp32 [sender][column][128 rows];
// a CTA finishes every parts-th column, so at most bn + 7 columns arrive). Outside the ring: a peer may be done, and sending,
// while this CTA's copies are still landing in its stages.
__host__ __device__ constexpr int recv_bytes(bool swap, int bn) { return swap ? (bn + 8) * kRowsA * 4 : 0; }
constexpr int kMaxStages = 12;
constexpr int64_t kCounterHeaderBytes = 64 * 1024;   // arrival counters of the feature tiles (stream-K), zero between launches

__host__ __device__ constexpr int stage_bytes(int bn) { return kRowsA * kBlockK * 2 + bn * kBlockK * 2; }
__host__ __device__ constexpr int ring_budget(bool swap, int bn) {
  return kSmemBudget < kSmemLimit - recv_bytes(swap, bn) ? kSmemBudget : kSmemLimit - recv_bytes(swap, bn);
}
__host__ __device__ constexpr int num_stages(bool swap, int bn) {
  return ring_budget(swap, bn) / stage_bytes(bn) < kMaxStages ? ring_budget(swap, bn) / stage_bytes(bn) : kMaxStages;
}
__host__ __device__ constexpr int smem_bytes(bool swap, int bn) {
  return num_stages(swap, bn) * stage_bytes(bn) + 1024 /* align */ + 512 /* barriers */ + recv_bytes(swap, bn);
}
// CTA pairs (many rows, 256-feature tiles): a stage holds this CTA's 128 token rows and ITS HALF of the 256 weight rows
constexpr int kBandM = 8;              // token tiles per band of the pairs' tile order
constexpr int kPairStageBytes = 2 * kRowsA * kBlockK * 2;
constexpr int kPairStages = 7;           // 224 KB of stages + barriers: all the shared memory a CTA may have (227 KB); 1.9 us of MMA work in flight
constexpr int kPairSmemBytes = kPairStages * kPairStageBytes + 1024 + 512;
__host__ __device__ constexpr uint32_t tmem_cols(int bn) { return 2 * bn < 32 ? 32u : static_cast<uint32_t>(2 * bn); }

struct Args {
  void* out; const void* bias;
  float* partials;       // shared tiles: [2 * grid][bn][128] fp32
  int* tile_counters;    // shared tiles: arrival counters, zero on entry, zero on exit
  int32_t* status;
  long long* trace;      // unused; the shared bounded-wait helper expects the member
  int64_t out_stride;    // elements
  int64_t m, n, k;
  int kb_total;          // k-blocks of 64
  int m_tiles, n_tiles;  // tiles along tokens / features
  int whole_tiles;       // tiles [0, whole_tiles) run whole, round-robin over the CTAs (always 0 with few rows)
  int64_t units;         // (tile, k-block) units of the remaining tiles, dealt evenly over the first sk_grid CTAs
  int sk_grid;           // CTAs that take a share of those units (<= gridDim.x, <= units): each owns at least one unit
  int cluster_parts;     // > 1: launched as thread-block clusters of this many CTAs; the CTAs of a cluster split the k-blocks of ONE
                         // feature tile and add their accumulators through distributed shared memory (few rows, few tiles)
  int epilogue;
  int weights_ahead;     // the weight copies of the first pipeline stages may be issued before the predecessor kernel has finished
                         // (the caller vouches that no kernel still in flight on the stream writes the weight matrix)
};

__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, uint64_t* bar, void* dst, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_cols(uint32_t* dst_smem, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)), "r"(cols) : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

// ---- thread-block cluster helpers ----
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {   // every thread of every CTA of the cluster
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// ---- CTA pairs: one tcgen05.mma over two SMs (cta_group::2), issued by the CTA of even rank ----
__device__ __forceinline__ uint32_t peer_addr(const void* local_smem, uint32_t cta) {   // the same offset in the CTA of rank `cta`
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local_smem)), "r"(cta));
  return remote;
}
// tile → this CTA's shared memory; the bytes are counted on a barrier that may live in the other CTA of the pair
__device__ __forceinline__ void tma_load_2d_pair(const CUtensorMap* map, uint32_t bar_cluster_addr, void* dst, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_cols_pair(uint32_t* dst_smem, uint32_t cols) {   // the same warp of BOTH CTAs
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)), "r"(cols) : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
// D[tmem of both CTAs, 256 rows] (+)= A[128 rows in each CTA's shared memory] * B[half of the N rows in each CTA's]
__device__ __forceinline__ void umma_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}
// one arrival, once every MMA issued so far has completed, on the barrier at this cluster address (either CTA of the pair)
__device__ __forceinline__ void umma_commit_pair(uint32_t bar_cluster_addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster_addr) : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster_addr) : "memory");
}

// `bytes` (a multiple of 16) from this CTA's shared memory to the same offset as `dst_local` in the CTA of rank `cta`, counted
// on the mbarrier at the offset of `bar_local` there (asynchronous copy between the shared memories of a cluster)
__device__ __forceinline__ void bulk_copy_to_peer(void* dst_local, const void* src, uint32_t bytes, uint64_t* bar_local, uint32_t cta) {
  uint32_t dst, bar;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(dst) : "r"(smem_u32(dst_local)), "r"(cta));
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(bar) : "r"(smem_u32(bar_local)), "r"(cta));
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(dst), "r"(smem_u32(src)), "r"(bytes), "r"(bar) : "memory");
}
__device__ __forceinline__ void cluster_sync_relaxed() {   // execution barrier only: orders no memory accesses
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}

// One piece of work of a CTA: k-blocks [kb0, kb1) of the tile at (a_row0, b_row0).
struct Segment {
  int a_row0, b_row0;   // first row of the A / B tile in its tensor
  int kb0, kb1;
  int shared_tile;      // index among the shared (stream-K) tiles: arrival counter; -1 for a whole tile
  bool partial;         // the tile's k-blocks are shared with other CTAs
};

// Stream-K bookkeeping: unit u = (shared tile, k-block); CTA c owns units [c*U/G, (c+1)*U/G).
__device__ __forceinline__ int64_t sk_first_unit(int64_t c, int64_t units, int64_t grid) { return c * units / grid; }
__device__ __forceinline__ int sk_cta_of(int64_t unit, int64_t units, int64_t grid) {
  return static_cast<int>(((unit + 1) * grid + units - 1) / units - 1);
}

// A CTA's list of segments: first its whole tiles (tile = blockIdx + i * grid: concurrent CTAs work on neighbouring tiles,
// which share a weight tile through L2), then its share of the (tile, k-block) units of the remaining tiles.
template <bool kSwap, int kBN, bool kPair = false>
struct Schedule {
  int64_t tile;             // next whole tile
  int64_t cursor, end;      // unit range of the shared tiles
  __device__ __forceinline__ void init(const Args& a) {
    tile = kPair ? blockIdx.x >> 1 : blockIdx.x;      // a pair of CTAs walks the 256-token tiles together
    cursor = end = 0;
    if (a.cluster_parts > 1) {          // one segment: this CTA's share of the k-blocks of tile blockIdx / parts
      const int64_t p = blockIdx.x % a.cluster_parts;
      cursor = p * a.kb_total / a.cluster_parts;
      end = (p + 1) * a.kb_total / a.cluster_parts;
      return;
    }
    const int64_t owner = kPair ? blockIdx.x >> 1 : blockIdx.x;     // pairs: both CTAs work the same unit range, each on its rows
    if (owner < a.sk_grid) {
      cursor = sk_first_unit(owner, a.units, a.sk_grid);
      end = sk_first_unit(owner + 1, a.units, a.sk_grid);
    }
  }
  __device__ __forceinline__ void place(const Args& a, int64_t t, Segment& s) const {
    if (kSwap) {
      s.a_row0 = static_cast<int>(t) * kRowsA;   // weight rows; all tokens (M <= kBN) are the B side
      s.b_row0 = 0;
    } else if (kPair) {
      // Bands of at most kBandM token tiles (all bands about equally tall), each swept feature tile by feature tile with the band's token tiles adjacent: the pairs
      // that run at the same time cover a roughly square patch (8 token tiles x 9 feature tiles on 74 pairs), so a tile of
      // either operand that one pair brings into L2 serves as many others as possible (a long K makes either operand larger
      // than L2: what is not shared between concurrent pairs is read from HBM again).
      const int n_bands = (a.m_tiles + kBandM - 1) / kBandM;
      const int tall = (a.m_tiles + n_bands - 1) / n_bands;                    // 17 token tiles: bands of 6, 6 and 5
      const int band = static_cast<int>(t / (static_cast<int64_t>(tall) * a.n_tiles));
      const int m0 = band * tall;
      const int rows = a.m_tiles - m0 < tall ? a.m_tiles - m0 : tall;          // token tiles of this band (the last may be shorter)
      const int in_band = static_cast<int>(t - static_cast<int64_t>(band) * tall * a.n_tiles);
      s.a_row0 = (m0 + in_band % rows) * (2 * kRowsA) + static_cast<int>(blockIdx.x & 1) * kRowsA;   // this CTA's half
      s.b_row0 = (in_band / rows) * kBN;      // all 256 weight rows of the tile (the accumulator's columns)
    } else {
      s.a_row0 = static_cast<int>(t % a.m_tiles) * kRowsA;   // tokens, fastest
      s.b_row0 = static_cast<int>(t / a.m_tiles) * kBN;      // weight rows
    }
  }
  __device__ __forceinline__ bool next(const Args& a, Segment& s) {
    if (a.cluster_parts > 1) {
      if (cursor >= end) return false;
      place(a, blockIdx.x / a.cluster_parts, s);
      s.kb0 = static_cast<int>(cursor); s.kb1 = static_cast<int>(end); s.shared_tile = -1; s.partial = false;
      cursor = end;
      return true;
    }
    if (tile < a.whole_tiles) {
      place(a, tile, s);
      s.kb0 = 0; s.kb1 = a.kb_total; s.shared_tile = -1; s.partial = false;
      tile += kPair ? gridDim.x >> 1 : gridDim.x;
      return true;
    }
    if (cursor >= end) return false;
    const int st = static_cast<int>(cursor / a.kb_total);
    const int64_t t0 = static_cast<int64_t>(st) * a.kb_total;
    const int64_t stop = end < t0 + a.kb_total ? end : t0 + a.kb_total;
    place(a, a.whole_tiles + st, s);
    s.shared_tile = st;
    s.kb0 = static_cast<int>(cursor - t0);
    s.kb1 = static_cast<int>(stop - t0);
    s.partial = !(s.kb0 == 0 && s.kb1 == a.kb_total);
    cursor = stop;
    return true;
  }
};

template <typename T>
__device__ __forceinline__ float round_to(float v) { return to_f32<T>(from_f32<T>(v)); }

// silu(gate) * up with the rounding of the unfused path: the projection output is rounded to T, silu is evaluated in fp32
// and rounded to T, the product is rounded to T.
template <typename T>
__device__ __forceinline__ T silu_mul(float gate_acc, float up_acc) {
  const float g = round_to<T>(gate_acc), u = round_to<T>(up_acc);
  const float act = round_to<T>(g / (1.f + expf(-g)));
  return from_f32<T>(act * u);
}
template <typename T>
__device__ __forceinline__ uint32_t pack2(T lo, T hi) {
  return static_cast<uint32_t>(*reinterpret_cast<uint16_t*>(&lo)) | (static_cast<uint32_t>(*reinterpret_cast<uint16_t*>(&hi)) << 16);
}

constexpr int kChunk = 16;   // accumulator columns handled at a time by an epilogue thread

template <bool kSwap, int kBN, typename T, bool kPair = false>
__global__ void __launch_bounds__(kThreads, 1)
linear_sm100_kernel(const __grid_constant__ CUtensorMap a_map, const __grid_constant__ CUtensorMap b_map, const Args a) {
  static_assert(!kPair || (!kSwap && kBN == 256), "CTA pairs serve the 256-feature tiles of the many-row plan");
  constexpr int kStages = kPair ? kPairStages : num_stages(kSwap, kBN);
  constexpr int kStageBytes = kPair ? kPairStageBytes : stage_bytes(kBN);
  constexpr int kABytes = kRowsA * kBlockK * 2;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* full = bars;                    // [kStages] TMA landed
  uint64_t* empty = bars + kStages;         // [kStages] MMAs that read the stage are done
  uint64_t* acc_full = bars + 2 * kStages;  // [2] accumulator complete
  uint64_t* acc_empty = acc_full + 2;       // [2] accumulator drained (one arrival per epilogue warp; pairs: of both CTAs, on the leader's)
  uint64_t* epi_all = acc_empty + 2;        // kEpiThreads arrivals: every epilogue thread published its partial
  uint64_t* epi_go = epi_all + 1;           // 1 arrival: the verdict "this CTA reduces the tile" is in shared memory
  uint64_t* recv_bar = epi_go + 1;          // cluster reduction: 128 arrivals per CTA of the cluster, every share has landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* reduce_flag = abort_flag + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (warp == 1) {
    if (lane == 0) {
      for (int i = 0; i < kStages; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
      for (int i = 0; i < 2; ++i) { mbar_init(&acc_full[i], 1); mbar_init(&acc_empty[i], (kPair ? 2 : 1) * (kEpiThreads / 32)); }   // every epilogue warp (pairs: of both CTAs)
      mbar_init(epi_all, kEpiThreads);
      mbar_init(epi_go, 1);
      mbar_init(recv_bar, 1);
      abort_flag[0] = 0;
      fence_barrier_init();
      if (kSwap && a.cluster_parts > 1) {
        // cluster reduction: this CTA finishes the token columns rank, rank + parts, ... and expects that many 512-byte
        // columns from every CTA of the cluster (its own share included)
        const int n_cols = static_cast<int>(a.m < kBN ? a.m : kBN), rank = static_cast<int>(cluster_ctarank());
        const int my_cols = n_cols > rank ? (n_cols - 1 - rank) / a.cluster_parts + 1 : 0;
        mbar_expect_tx(recv_bar, static_cast<uint32_t>(a.cluster_parts * my_cols * kRowsA * 4));
      }
    }
    __syncwarp();
    if (kPair) tmem_alloc_cols_pair(tmem_slot, tmem_cols(kBN));
    else tmem_alloc_cols(tmem_slot, tmem_cols(kBN));
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // the peers' receive barriers exist before anyone can arrive on them (ahead of the dependency wait: the CTAs of a cluster
  // start together, and the predecessor kernel is still finishing)
  if ((kSwap && a.cluster_parts > 1) || kPair) cluster_sync_all();
  // pairs: the CTA of even rank (the leader) owns the barriers that say "stage filled" and "accumulator drained", and issues
  // every MMA; each CTA owns its "stage free" and "accumulator complete" barriers, on which the leader's commits arrive
  const uint32_t pair_rank = kPair ? cluster_ctarank() : 0u;

  Schedule<kSwap, kBN, kPair> sched;
  sched.init(a);
  Segment seg;

  // Barriers and TMEM are set up; from here on the kernel reads what its predecessor wrote, so every thread waits for the
  // predecessor's completion first. The one exception is the producer thread when the weights are known to be at rest: it
  // first fills the pipeline with the WEIGHT halves of the first stages, so that the weight stream of this kernel starts while
  // the kernel before it is still finishing, and issues the activation halves after its wait.
  const bool producer_thread = warp == 0 && lane == 0;
  if (!producer_thread) {
    grid_dependency_wait();
    grid_launch_dependents();
  }

  if (warp == 0) {
    // =========================== TMA producer ===========================
    if (lane == 0) {
      int ahead = 0;                                  // stages whose weight half is already on its way
      if (kSwap && a.weights_ahead) {
        Schedule<kSwap, kBN, kPair> peek = sched;
        Segment s0;
        const int limit = a.weights_ahead < kStages ? a.weights_ahead : kStages;
        while (ahead < limit && peek.next(a, s0)) {
          for (int kb = s0.kb0; kb < s0.kb1 && ahead < limit; ++kb, ++ahead) {
            mbar_expect_tx(&full[ahead], kStageBytes);
            tma_load_2d(&a_map, &full[ahead], smem + ahead * kStageBytes, kb * kBlockK, s0.a_row0);
          }
        }
      }
      grid_dependency_wait();
      grid_launch_dependents();
      int stage = 0; uint32_t phase = 0;
      int step = 0;
      bool ok = true;
      while (ok && sched.next(a, seg)) {
        for (int kb = seg.kb0; kb < seg.kb1 && ok; ++kb, ++step) {
          uint8_t* sa = smem + stage * kStageBytes;
          if (step < ahead) {                         // first lap: the stage is free and its weight half was issued above
            tma_load_2d(&b_map, &full[stage], sa + kABytes, kb * kBlockK, seg.b_row0);
          } else if (kPair) {
            ok = mbar_wait(&empty[stage], phase ^ 1, abort_flag, a);
            if (!ok) break;
            // both CTAs' copies of the stage are counted on the leader's barrier, which expects the bytes of both
            if (pair_rank == 0) mbar_expect_tx(&full[stage], 2 * kStageBytes);
            const uint32_t bar = peer_addr(&full[stage], 0);
            tma_load_2d_pair(&a_map, bar, sa, kb * kBlockK, seg.a_row0);
            tma_load_2d_pair(&b_map, bar, sa + kABytes, kb * kBlockK, seg.b_row0 + static_cast<int>(pair_rank) * (kBN / 2));
          } else {
            ok = mbar_wait(&empty[stage], phase ^ 1, abort_flag, a);   // a fresh barrier passes the first lap
            if (!ok) break;
            mbar_expect_tx(&full[stage], kStageBytes);
            tma_load_2d(&a_map, &full[stage], sa, kb * kBlockK, seg.a_row0);
            tma_load_2d(&b_map, &full[stage], sa + kABytes, kb * kBlockK, seg.b_row0);
          }
          if (++stage == kStages) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) {   // the CTA is abandoning its result: give copies in flight a bounded moment to land
        const long long t0 = clock64();
        while (clock64() - t0 < 200000) { }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // =========================== MMA issuer ===========================
    if (lane == 0 && pair_rank == 0) {
      // pairs: M = 256 (bits 24-28 hold M / 16), N = 256; one instruction covers both CTAs' token rows
      const uint32_t idesc = kPair ? (make_idesc(kBf16, false, kBN) & ~(0x1fu << 24)) | ((2u * kRowsA >> 4) << 24) : make_idesc(kBf16, false, kBN);
      int stage = 0; uint32_t phase = 0;
      int n_seg = 0;
      bool ok = true;
      while (ok && sched.next(a, seg)) {
        const int acc = n_seg & 1;
        const uint32_t acc_phase = (n_seg >> 1) & 1;
        ++n_seg;
        ok = mbar_wait(&acc_empty[acc], acc_phase ^ 1, abort_flag, a);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * kBN);
        for (int kb = seg.kb0; kb < seg.kb1 && ok; ++kb) {
          ok = mbar_wait(&full[stage], phase, abort_flag, a);
          if (!ok) break;
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * kStageBytes), sb = sa + kABytes;
#pragma unroll
          for (int kk = 0; kk < kBlockK / 16; ++kk) {
            if (kPair) umma_ss_pair(d, desc_kmajor_sw128(sa + kk * 32), desc_kmajor_sw128(sb + kk * 32), idesc, (kb > seg.kb0 || kk > 0) ? 1u : 0u);
            else umma_ss(d, desc_kmajor_sw128(sa + kk * 32), desc_kmajor_sw128(sb + kk * 32), idesc, (kb > seg.kb0 || kk > 0) ? 1u : 0u);
          }
          if (kPair) { umma_commit_pair(smem_u32(&empty[stage])); umma_commit_pair(peer_addr(&empty[stage], 1)); }
          else umma_commit(&empty[stage]);
          if (++stage == kStages) { stage = 0; phase ^= 1; }
        }
        if (ok) {
          if (kPair) { umma_commit_pair(smem_u32(&acc_full[acc])); umma_commit_pair(peer_addr(&acc_full[acc], 1)); }
          else umma_commit(&acc_full[acc]);
        }
      }
    }
    __syncwarp();
  } else {
    // =========================== epilogue: warps 2-9, thread = accumulator row, two warps per row ===========================
    const int quarter = warp & 3;                       // the TMEM lanes a warp may read: 32 * (warp id mod 4)
    const int r = quarter * 32 + lane;                  // accumulator row
    const int et = threadIdx.x - kEpiWarp0 * 32;        // 0..255
    const int half = (warp - kEpiWarp0) >> 2;           // chunks half, half + 2, ... of the accumulator's columns
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    T* out = reinterpret_cast<T*>(a.out);
    const T* bias = reinterpret_cast<const T*>(a.bias);
    const bool silu = a.epilogue == PDLLM_EPI_SILU_MUL;
    // accumulator columns that carry data: the tokens (few rows: out^T) or the whole feature tile
    const int n_cols = kSwap ? static_cast<int>(a.m < kBN ? a.m : kBN) : kBN;
    int n_seg = 0;
    uint32_t epi_phase = 0;
    bool ok = true;
    while (ok && sched.next(a, seg)) {
      const int acc = n_seg & 1;
      const uint32_t acc_phase = (n_seg >> 1) & 1;
      ++n_seg;
      // (sleeping between polls: 256 threads wait here for a whole main loop, tens of microseconds on the many-row shapes,
      // and the part runs against its power limit there)
      ok = mbar_wait<true>(&acc_full[acc], acc_phase, abort_flag, a);
      if (!ok) break;
      tc_fence_after();
      const uint32_t t_acc = tmem_base + lane_base + static_cast<uint32_t>(acc * kBN);

      // Finished values of accumulator columns [c0, c0 + 16) of row r → output.
      //   few rows:  row r = feature n, column = token: 2-byte stores, a warp covers 32 consecutive features of one token;
      //   many rows: row r = token, columns = features: 32 contiguous bytes per thread.
      const int64_t row_id = static_cast<int64_t>(seg.a_row0) + r;     // feature (few rows) or token (many rows)
      float bias_r = 0.f;
      if (kSwap && bias != nullptr && row_id < a.n) bias_r = to_f32<T>(bias[row_id]);
      auto store_chunk = [&](int c0, const float* v) {
        if (kSwap) {
          if (silu) {
            // all sixteen activations first, as independent chains (one warp per scheduler: nothing else hides the latency
            // of the exponential and the division), then the stores
            T res[kChunk];
#pragma unroll
            for (int i = 0; i < kChunk; ++i) {
              const float other = __shfl_xor_sync(0xffffffffu, v[i], 1);
              res[i] = silu_mul<T>(v[i], other);
            }
            if ((lane & 1) == 0 && row_id + 1 < a.n) {
#pragma unroll
              for (int i = 0; i < kChunk; ++i) {
                if (c0 + i < n_cols) out[static_cast<int64_t>(c0 + i) * a.out_stride + (row_id >> 1)] = res[i];
              }
            }
          } else if (row_id < a.n) {
#pragma unroll
            for (int i = 0; i < kChunk; ++i) {
              if (c0 + i < n_cols) out[static_cast<int64_t>(c0 + i) * a.out_stride + row_id] = from_f32<T>(v[i] + bias_r);
            }
          }
        } else {
          const int64_t n0 = static_cast<int64_t>(seg.b_row0) + c0;
          if (row_id >= a.m || n0 >= a.n) return;
          if (silu) {
            T* dst = out + row_id * a.out_stride + (n0 >> 1);
            if (n0 + kChunk <= a.n) {
              uint32_t p[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) p[i] = pack2<T>(silu_mul<T>(v[4 * i], v[4 * i + 1]), silu_mul<T>(v[4 * i + 2], v[4 * i + 3]));
              *reinterpret_cast<uint4*>(dst) = make_uint4(p[0], p[1], p[2], p[3]);
            } else {
              for (int i = 0; i < kChunk / 2 && n0 + 2 * i + 1 < a.n; ++i) dst[i] = silu_mul<T>(v[2 * i], v[2 * i + 1]);
            }
          } else {
            T* dst = out + row_id * a.out_stride + n0;
            if (n0 + kChunk <= a.n) {
              uint32_t p[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                float x0 = v[2 * i], x1 = v[2 * i + 1];
                if (bias != nullptr) { x0 += to_f32<T>(bias[n0 + 2 * i]); x1 += to_f32<T>(bias[n0 + 2 * i + 1]); }
                p[i] = pack2<T>(from_f32<T>(x0), from_f32<T>(x1));
              }
              uint4* d4 = reinterpret_cast<uint4*>(dst);
              d4[0] = make_uint4(p[0], p[1], p[2], p[3]);
              d4[1] = make_uint4(p[4], p[5], p[6], p[7]);
            } else {
              for (int i = 0; i < kChunk && n0 + i < a.n; ++i) dst[i] = from_f32<T>(v[i] + (bias != nullptr ? to_f32<T>(bias[n0 + i]) : 0.f));
            }
          }
        }
      };

      if (kSwap && a.cluster_parts > 1) {
        // The CTAs of the cluster hold shares of ONE tile; the CTA of rank p finishes the token columns p, p + parts, ....
        // Every CTA lays its accumulator out by finisher in its own (by now idle) pipeline stages — fp32
        // [finisher][column][128 rows] — and ONE thread sends each finisher its columns with an asynchronous copy between
        // shared memories that counts on the finisher's barrier. A finisher adds the shares out of its own receive buffer
        // ([sender][column][128 rows], outside the ring: a fast peer sends while this CTA's stages are still in use).
        // Nobody waits for a slower peer except for the shares it has to add.
        const int parts = a.cluster_parts;
        const int rank = static_cast<int>(cluster_ctarank());
        const int per = (n_cols + parts - 1) / parts;       // columns of the largest share
        float* send = reinterpret_cast<float*>(smem);
        float* recv = reinterpret_cast<float*>(smem + kStages * kStageBytes + 512);
#pragma unroll 1
        for (int c0 = half * kChunk; c0 < n_cols; c0 += 2 * kChunk) {
          uint32_t raw[kChunk];
          tc::tmem_ld16(t_acc + c0, raw);
          tc_wait_ld();
          int dst = c0 % parts, lc = c0 / parts;
#pragma unroll
          for (int i = 0; i < kChunk; ++i) {
            if (c0 + i < n_cols) send[(dst * per + lc) * kRowsA + r] = __uint_as_float(raw[i]);
            if (++dst == parts) { dst = 0; ++lc; }
          }
        }
        tc_fence_before();
        tc::fence_proxy_async();                              // the copies below read what this thread just wrote
        asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
        if (lane == 0) mbar_arrive(&acc_empty[acc]);
        if (et == 0) {
          for (int p = 0; p < parts; ++p) {
            const int cols_p = n_cols > p ? (n_cols - 1 - p) / parts + 1 : 0;
            if (cols_p > 0)
              bulk_copy_to_peer(recv + rank * per * kRowsA, send + p * per * kRowsA, static_cast<uint32_t>(cols_p * kRowsA * 4), recv_bar, static_cast<uint32_t>(p));
          }
        }
        ok = mbar_wait(recv_bar, 0, abort_flag, a);
        if (!ok) break;
        // shares added in rank order: the result does not depend on timing. All loads of a column group first.
        const int my_cols = n_cols > rank ? (n_cols - 1 - rank) / parts + 1 : 0;
#pragma unroll 1
        for (int l0 = half * 4; l0 < my_cols; l0 += 8) {
          float v[8][4];
#pragma unroll
          for (int p = 0; p < 8; ++p) {
#pragma unroll
            for (int i = 0; i < 4; ++i) v[p][i] = (p < parts && l0 + i < my_cols) ? recv[(p * per + l0 + i) * kRowsA + r] : 0.f;
          }
          float sum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int p = 0; p < 8; ++p) {
#pragma unroll
            for (int i = 0; i < 4; ++i) sum[i] += v[p][i];
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            if (l0 + i >= my_cols) break;             // uniform across the warp
            const int j = (l0 + i) * parts + rank;
            if (silu) {
              const float other = __shfl_xor_sync(0xffffffffu, sum[i], 1);
              if ((lane & 1) == 0 && row_id + 1 < a.n) out[static_cast<int64_t>(j) * a.out_stride + (row_id >> 1)] = silu_mul<T>(sum[i], other);
            } else if (row_id < a.n) {
              out[static_cast<int64_t>(j) * a.out_stride + row_id] = from_f32<T>(sum[i] + bias_r);
            }
          }
        }
      } else if (!seg.partial) {
#pragma unroll 1
        for (int c0 = half * kChunk; c0 < n_cols; c0 += 2 * kChunk) {
          uint32_t raw[kChunk];
          tc::tmem_ld16(t_acc + c0, raw);
          tc_wait_ld();
          float v[kChunk];
#pragma unroll
          for (int i = 0; i < kChunk; ++i) v[i] = __uint_as_float(raw[i]);
          store_chunk(c0, v);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (kPair) mbar_arrive_cluster(peer_addr(&acc_empty[acc], 0));   // the leader waits for both CTAs' epilogues
          else mbar_arrive(&acc_empty[acc]);
        }
      } else {
        // This CTA holds only some k-blocks of the tile: publish its share as fp32 [128 rows][kBN columns]; slot 0 = the first
        // shared tile of the CTA's unit range, slot 1 = its last.
        // (pairs: the unit ranges belong to pairs; each CTA publishes, counts and reduces its own 128 rows independently)
        const int64_t owner = kPair ? blockIdx.x >> 1 : blockIdx.x;
        const int side = kPair ? static_cast<int>(blockIdx.x & 1) : 0;
        const int first_st = static_cast<int>(sk_first_unit(owner, a.units, a.sk_grid) / a.kb_total);
        float* mine = a.partials + (static_cast<int64_t>(blockIdx.x) * 2 + (seg.shared_tile == first_st ? 0 : 1)) * (kBN * kRowsA) + r * kBN;
#pragma unroll 1
        for (int c0 = half * kChunk; c0 < n_cols; c0 += 2 * kChunk) {
          uint32_t raw[kChunk];
          tc::tmem_ld16(t_acc + c0, raw);
          tc_wait_ld();
          uint4* dst = reinterpret_cast<uint4*>(mine + c0);
#pragma unroll
          for (int i = 0; i < kChunk / 4; ++i) dst[i] = make_uint4(raw[4 * i], raw[4 * i + 1], raw[4 * i + 2], raw[4 * i + 3]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (kPair) mbar_arrive_cluster(peer_addr(&acc_empty[acc], 0));
          else mbar_arrive(&acc_empty[acc]);
        }
        __threadfence();
        mbar_arrive(epi_all);
        const int64_t t0 = static_cast<int64_t>(seg.shared_tile) * a.kb_total;
        if (et == 0) {
          ok = mbar_wait(epi_all, epi_phase, abort_flag, a);
          if (ok) {
            const int parts = sk_cta_of(t0 + a.kb_total - 1, a.units, a.sk_grid) - sk_cta_of(t0, a.units, a.sk_grid) + 1;
            int* counter = &a.tile_counters[kPair ? 2 * seg.shared_tile + side : seg.shared_tile];
            const int prev = atomicAdd(counter, 1);
            const int last = prev == parts - 1 ? 1 : 0;
            if (last) *counter = 0;      // every share has arrived: ready for the next launch
            reduce_flag[0] = last;
            mbar_arrive(epi_go);
          }
        }
        ok = mbar_wait(epi_go, epi_phase, abort_flag, a);
        epi_phase ^= 1;
        if (!ok) break;
        if (reduce_flag[0]) {
          __threadfence();
          // Shares are added in CTA order c_first..c_last, whoever reduces. Every CTA after the first starts inside this
          // tile, so the tile is its first (slot 0); for the first CTA that holds only when its range starts exactly here.
          // Four shares x 16 columns of a row are in flight per thread (sixteen 16-byte loads), then added in order.
          const int c_first = sk_cta_of(t0, a.units, a.sk_grid), c_last = sk_cta_of(t0 + a.kb_total - 1, a.units, a.sk_grid);
          const int first_slot = sk_first_unit(c_first, a.units, a.sk_grid) == t0 ? 0 : 1;
          constexpr int kBatch = 4;
#pragma unroll 1
          for (int c0 = half * kChunk; c0 < n_cols; c0 += 2 * kChunk) {
            float sum[kChunk];
#pragma unroll
            for (int i = 0; i < kChunk; ++i) sum[i] = 0.f;
#pragma unroll 1
            for (int cb = c_first; cb <= c_last; cb += kBatch) {
              float4 v[kBatch][kChunk / 4];
#pragma unroll
              for (int p = 0; p < kBatch; ++p) {
                const int c = cb + p;
                const float4* part = reinterpret_cast<const float4*>(
                    a.partials + ((kPair ? static_cast<int64_t>(c) * 2 + side : static_cast<int64_t>(c)) * 2 + (c == c_first ? first_slot : 0)) * (kBN * kRowsA) + r * kBN + c0);
#pragma unroll
                for (int i = 0; i < kChunk / 4; ++i) v[p][i] = c <= c_last ? __ldcg(part + i) : make_float4(0.f, 0.f, 0.f, 0.f);
              }
#pragma unroll
              for (int p = 0; p < kBatch; ++p) {
#pragma unroll
                for (int i = 0; i < kChunk / 4; ++i) {
                  sum[4 * i] += v[p][i].x; sum[4 * i + 1] += v[p][i].y; sum[4 * i + 2] += v[p][i].z; sum[4 * i + 3] += v[p][i].w;
                }
              }
            }
            store_chunk(c0, sum);
          }
        }
      }
    }
  }

  // ---- teardown ----
  // A CTA of a cluster leaves only when every peer holds all its shares: the copies out of this CTA's shared memory are then
  // complete. (Execution barrier only: nobody has to see this CTA's output stores before it may go.)
  if (kSwap && a.cluster_parts > 1) cluster_sync_relaxed();
  // Pairs: the leader's MMAs read the other CTA's shared memory and write its TMEM, the other CTA's copies and arrivals
  // land on the leader's barriers: neither leaves, nor frees TMEM, before both are done.
  if (kPair) { tc_fence_before(); cluster_sync_all(); }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if (kPair) tmem_dealloc_pair(tmem_base, tmem_cols(kBN));
    else tc::tmem_dealloc(tmem_base, tmem_cols(kBN));
  }
}

// ---- host side ---------------------------------------------------------------------------------------------
struct Plan {
  bool swap;
  bool pair;      // many rows: 256 x 256 tiles worked by pairs of CTAs (one MMA over two SMs)
  int bn;         // B-tile rows: token tile (few rows) or feature tile (many rows)
  int m_tiles, n_tiles, kb_total;
  int whole_tiles;   // tiles that run whole, round-robin
  int shared_tiles;  // tiles whose k-blocks are dealt over all CTAs
  int64_t units;     // shared_tiles * kb_total
  int sk_grid;       // CTAs that share those units
  int cluster_parts; // > 1: clusters of this many CTAs per feature tile (few rows, few tiles)
  int grid;
};

// PDLLM_GEMM_PAIRS=0: every many-row tile in one CTA (for comparisons)
inline bool pairs_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("PDLLM_GEMM_PAIRS");
    return !(v != nullptr && v[0] == '0');
  }();
  return on;
}

inline Plan make_plan(int64_t m, int64_t n, int64_t k) {
  Plan pl;
  pl.pair = false;
  const int sms = sm_count();
  pl.kb_total = static_cast<int>((k + kBlockK - 1) / kBlockK);
  pl.swap = m <= 128;
  int64_t tiles, sk_ctas = 0;
  if (pl.swap) {
    // bound by streaming the weights: every k-block of every feature tile is a unit, all dealt evenly
    pl.bn = m <= 16 ? 16 : m <= 32 ? 32 : m <= 64 ? 64 : 128;
    pl.m_tiles = 1;
    pl.n_tiles = static_cast<int>((n + kRowsA - 1) / kRowsA);
    tiles = pl.n_tiles;
    pl.whole_tiles = 0;
  } else {
    pl.m_tiles = static_cast<int>((m + kRowsA - 1) / kRowsA);
    const int64_t tiles256 = static_cast<int64_t>(pl.m_tiles) * ((n + 255) / 256);
    // Narrower tiles when wide ones would leave SMs without work. (Keeping the wide tile and dealing the (tile, k-block) units of
    // ALL tiles over the SMs was measured at 512 rows: 3x slower — every CTA then trades a 128 KB fp32 partial through L2.)
    pl.bn = tiles256 >= sms ? 256 : 128;
    // (pairs also for fewer wide tiles than SMs when K is long: the tiles are then cut along K over the idle pairs — the down
    // projection at a few hundred rows, 28 tiles of 296 k-blocks)
    if ((pl.bn == 256 || pl.kb_total >= 128) && m >= 512 && pairs_enabled()) {
      pl.bn = 256;
      // Two CTAs per 256-token x 256-feature tile: each stages its 128 token rows and HALF of the weight rows, and one
      // tcgen05.mma (cta_group::2, M = 256) reads both shared memories — half the shared-memory traffic per flop of the
      // single-CTA 128 x 256 tile, and a ring of 6 stages instead of 4. Whole tiles only, dealt round-robin over the pairs.
      pl.pair = true;
      pl.m_tiles = static_cast<int>((m + 2 * kRowsA - 1) / (2 * kRowsA));
      pl.n_tiles = static_cast<int>((n + 255) / 256);
      tiles = static_cast<int64_t>(pl.m_tiles) * pl.n_tiles;
      pl.whole_tiles = static_cast<int>(tiles);
      pl.shared_tiles = 0; pl.units = 0; pl.sk_grid = 0; pl.cluster_parts = 1;
      const int64_t slots = sms / 2;
      // as with single CTAs: a last wave that fills less than three quarters of the pairs is cut along K, `parts` pairs per tile
      const int64_t rest_p = tiles % slots;
      if (rest_p > 0 && rest_p * 4 < slots * 3) {
        // (at least 32 k-blocks per share: a share costs a 128 KB fp32 partial per CTA through L2, measured to outweigh the
        // saved wave at K = 3584 and to pay at K = 18944)
        int64_t parts = slots / rest_p;
        if (parts > pl.kb_total / 32) parts = pl.kb_total / 32;
        if (parts >= 2 && rest_p * 2 * 4 <= kCounterHeaderBytes) {
          pl.whole_tiles = static_cast<int>(tiles - rest_p);
          pl.shared_tiles = static_cast<int>(rest_p);
          pl.units = rest_p * pl.kb_total;
          pl.sk_grid = static_cast<int>(rest_p * parts);
        }
      }
      const int64_t busy = pl.whole_tiles >= slots ? slots : (pl.whole_tiles > pl.sk_grid ? pl.whole_tiles : pl.sk_grid);
      pl.grid = static_cast<int>(2 * (busy < 1 ? 1 : busy));
      return pl;
    }
    pl.n_tiles = static_cast<int>((n + pl.bn - 1) / pl.bn);
    tiles = static_cast<int64_t>(pl.m_tiles) * pl.n_tiles;
    // Full waves of whole tiles. A last wave that fills less than three quarters of the SMs is cut along K instead: each of
    // its tiles goes to `parts` CTAs (at least 8 k-blocks each), so the tail of the kernel is a fraction of a tile long.
    pl.whole_tiles = static_cast<int>(tiles);
    const int64_t rest = tiles % sms;
    if (rest > 0 && rest * 4 < static_cast<int64_t>(sms) * 3) {
      int64_t parts = sms / rest;
      if (parts > pl.kb_total / 8) parts = pl.kb_total / 8;
      if (parts >= 2) {
        pl.whole_tiles = static_cast<int>(tiles - rest);
        sk_ctas = rest * parts;
      }
    }
  }
  pl.cluster_parts = 1;
  if (pl.swap && 2 * tiles <= sms) {
    // Fewer feature tiles than half the SMs (the QKV, O and down projections of a 7B model): a cluster of `parts` CTAs per
    // tile, each streaming 1/parts of the tile's k-blocks, summed through distributed shared memory — no workspace round
    // trip, no arrival counters. parts: as many as fill the SMs, at most 8 (the portable cluster size), at least 4 k-blocks each.
    int64_t parts = sms / tiles;
    if (parts > 8) parts = 8;
    if (parts > pl.kb_total / 4) parts = pl.kb_total / 4;
    if (parts >= 2) pl.cluster_parts = static_cast<int>(parts);
  }
  if (pl.cluster_parts > 1) {
    pl.whole_tiles = 0; pl.shared_tiles = 0; pl.units = 0; pl.sk_grid = 0;
    pl.grid = static_cast<int>(tiles) * pl.cluster_parts;
    return pl;
  }
  pl.shared_tiles = static_cast<int>(tiles - pl.whole_tiles);
  pl.units = static_cast<int64_t>(pl.shared_tiles) * pl.kb_total;
  if (pl.swap) sk_ctas = pl.units < sms ? pl.units : sms;
  pl.sk_grid = static_cast<int>(sk_ctas);
  int64_t grid = pl.whole_tiles >= sms ? sms : (pl.whole_tiles > sk_ctas ? pl.whole_tiles : sk_ctas);
  pl.grid = static_cast<int>(grid < 1 ? 1 : grid);
  return pl;
}

inline int64_t workspace_bytes(int64_t m, int64_t n, int64_t k) {
  if (m <= 0 || n <= 0) return 0;
  const Plan pl = make_plan(m, n, k);
  // a grid never exceeds the SM count; sized for it so that one workspace serves every layer of a model
  return kCounterHeaderBytes + static_cast<int64_t>(2) * sm_count() * pl.bn * kRowsA * 4;
}

template <bool kSwap, int kBN, typename T>
inline int launch_one(const CUtensorMap& a_map, const CUtensorMap& b_map, const Args& a, int grid, cudaStream_t stream) {
  auto* fn = linear_sm100_kernel<kSwap, kBN, T>;
  {
    static std::mutex mu;
    static bool done[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 0 || dev >= 64 || !done[dev]) {
      cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes(kSwap, kBN));
      if (e != cudaSuccess) return fail(static_cast<int>(e), "cudaFuncSetAttribute(linear): %s", cudaGetErrorString(e));
      if (dev >= 0 && dev < 64) done[dev] = true;
    }
  }
  if (a.cluster_parts > 1) {
    // All clusters of the launch must be resident at once (one CTA per SM, clusters packed per GPC): take the largest
    // cluster size, from the planned one down, for which the device says that many clusters fit; with none, one CTA per tile.
    const int tiles = grid / a.cluster_parts;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem_bytes(kSwap, kBN);
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;   // see launch_dependent(): start ahead of the predecessor's end
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    static std::mutex mu_fit;
    static int fits[64][9] = {};      // per device and cluster size: max resident clusters + 1 (0 = not asked yet)
    int dev = 0;
    cudaGetDevice(&dev);
    int parts = a.cluster_parts;
    for (; parts >= 2; --parts) {
      int n_fit = -1;
      {
        std::lock_guard<std::mutex> lock(mu_fit);
        if (dev >= 0 && dev < 64 && fits[dev][parts] > 0) n_fit = fits[dev][parts] - 1;
      }
      if (n_fit < 0) {
        cfg.gridDim = dim3(static_cast<unsigned>(tiles * parts), 1, 1);
        attr[0].val.clusterDim.x = static_cast<unsigned>(parts);
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess) { (void)cudaGetLastError(); n = 0; }
        n_fit = n;
        std::lock_guard<std::mutex> lock(mu_fit);
        if (dev >= 0 && dev < 64) fits[dev][parts] = n + 1;
      }
      if (n_fit >= tiles) break;
    }
    Args b = a;
    b.cluster_parts = parts >= 2 ? parts : 1;
    if (b.cluster_parts > 1) {
      cfg.gridDim = dim3(static_cast<unsigned>(tiles * b.cluster_parts), 1, 1);
      attr[0].val.clusterDim.x = static_cast<unsigned>(b.cluster_parts);
      cfg.numAttrs = dependent_launch_enabled() ? 2 : 1;
      cudaError_t e = cudaLaunchKernelEx(&cfg, fn, a_map, b_map, b);
      if (e != cudaSuccess) return fail(static_cast<int>(e), "linear_sm100_kernel (clusters of %d): %s", b.cluster_parts, cudaGetErrorString(e));
      return check_launch("linear_sm100_kernel");
    }
    // no cluster size fits: every tile whole in one CTA (no workspace needed)
    b.whole_tiles = tiles; b.units = 0; b.sk_grid = 0;
    (void)launch_dependent(fn, dim3(static_cast<unsigned>(tiles)), dim3(kThreads), smem_bytes(kSwap, kBN), stream, a_map, b_map, b);
    return check_launch("linear_sm100_kernel");
  }
  (void)launch_dependent(fn, dim3(static_cast<unsigned>(grid)), dim3(kThreads), smem_bytes(kSwap, kBN), stream, a_map, b_map, a);
  return check_launch("linear_sm100_kernel");
}

template <typename T>
inline int launch_pairs(const CUtensorMap& a_map, const CUtensorMap& b_map, const Args& a, int grid, cudaStream_t stream) {
  auto* fn = linear_sm100_kernel<false, 256, T, true>;
  {
    static std::mutex mu;
    static bool done[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 0 || dev >= 64 || !done[dev]) {
      cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kPairSmemBytes);
      if (e != cudaSuccess) return fail(static_cast<int>(e), "cudaFuncSetAttribute(linear, pairs): %s", cudaGetErrorString(e));
      if (dev >= 0 && dev < 64) done[dev] = true;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kPairSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = dependent_launch_enabled() ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, fn, a_map, b_map, a);
  if (e != cudaSuccess) return fail(static_cast<int>(e), "linear_sm100_kernel (CTA pairs): %s", cudaGetErrorString(e));
  return check_launch("linear_sm100_kernel");
}

template <typename T>
inline int launch_typed(const Plan& pl, const CUtensorMap& a_map, const CUtensorMap& b_map, const Args& a, cudaStream_t stream) {
  if (pl.pair) return launch_pairs<T>(a_map, b_map, a, pl.grid, stream);
  if (pl.swap) {
    switch (pl.bn) {
      case 16: return launch_one<true, 16, T>(a_map, b_map, a, pl.grid, stream);
      case 32: return launch_one<true, 32, T>(a_map, b_map, a, pl.grid, stream);
      case 64: return launch_one<true, 64, T>(a_map, b_map, a, pl.grid, stream);
      default: return launch_one<true, 128, T>(a_map, b_map, a, pl.grid, stream);
    }
  }
  if (pl.bn == 256) return launch_one<false, 256, T>(a_map, b_map, a, pl.grid, stream);
  return launch_one<false, 128, T>(a_map, b_map, a, pl.grid, stream);
}

// pipeline stages whose weight half is requested before the dependency wait (PDLLM_WEIGHTS_AHEAD overrides, for experiments)
inline int stages_ahead() {
  static const int n = [] {
    const char* v = std::getenv("PDLLM_WEIGHTS_AHEAD");
    return v != nullptr && v[0] != '\0' ? std::atoi(v) : 4;
  }();
  return n;
}

inline int launch(const void* x, int64_t x_stride, const void* w, int64_t w_stride, const void* bias, void* out, int64_t out_stride,
                  int64_t m, int64_t n, int64_t k, int dtype, int epilogue, void* workspace, int64_t ws_bytes, int workspace_zeroed,
                  int32_t* status, cudaStream_t stream) {
  const bool bf16 = dtype == PDLLM_BF16;
  const Plan pl = make_plan(m, n, k);
  CUtensorMap x_map, w_map;
  int rc;
  {
    uint64_t dims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(m)};
    uint64_t str[1] = {static_cast<uint64_t>(x_stride) * 2};
    uint32_t box[2] = {kBlockK, static_cast<uint32_t>(pl.swap ? pl.bn : kRowsA)};
    if ((rc = tc::encode_map(&x_map, bf16, x, 2, dims, str, box)) != 0) return rc;
  }
  {
    uint64_t dims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(n)};
    uint64_t str[1] = {static_cast<uint64_t>(w_stride) * 2};
    uint32_t box[2] = {kBlockK, static_cast<uint32_t>(pl.swap ? kRowsA : (pl.pair ? pl.bn / 2 : pl.bn))};   // pairs: each CTA copies its half
    if ((rc = tc::encode_map(&w_map, bf16, w, 2, dims, str, box)) != 0) return rc;
  }
  Args a;
  a.out = out; a.bias = bias; a.status = status; a.trace = nullptr;
  a.out_stride = out_stride; a.m = m; a.n = n; a.k = k;
  a.kb_total = pl.kb_total; a.m_tiles = pl.m_tiles; a.n_tiles = pl.n_tiles; a.whole_tiles = pl.whole_tiles; a.units = pl.units; a.sk_grid = pl.sk_grid; a.cluster_parts = pl.cluster_parts;
  a.epilogue = epilogue & 0xff;
  a.weights_ahead = (epilogue & PDLLM_LINEAR_WEIGHTS_AT_REST) ? stages_ahead() : 0;
  a.partials = nullptr; a.tile_counters = nullptr;
  if (pl.shared_tiles > 0) {
    const int64_t need = workspace_bytes(m, n, k);
    if (workspace == nullptr || ws_bytes < need)
      return fail(PDLLM_E_WORKSPACE, "linear needs %lld workspace bytes, got %lld", static_cast<long long>(need), static_cast<long long>(ws_bytes));
    if (static_cast<int64_t>(pl.shared_tiles) * 4 > kCounterHeaderBytes)
      return fail(PDLLM_E_UNSUPPORTED, "linear: %d shared tiles exceed the arrival-counter header", pl.shared_tiles);
    a.tile_counters = reinterpret_cast<int*>(workspace);
    a.partials = reinterpret_cast<float*>(static_cast<char*>(workspace) + kCounterHeaderBytes);
    if (!workspace_zeroed) {
      cudaError_t e = cudaMemsetAsync(a.tile_counters, 0, static_cast<size_t>(pl.shared_tiles) * (pl.pair ? 8 : 4), stream);
      if (e != cudaSuccess) return fail(static_cast<int>(e), "cudaMemsetAsync(linear counters): %s", cudaGetErrorString(e));
    }
  }
  const CUtensorMap& a_map = pl.swap ? w_map : x_map;
  const CUtensorMap& b_map = pl.swap ? x_map : w_map;
  return bf16 ? launch_typed<__nv_bfloat16>(pl, a_map, b_map, a, stream) : launch_typed<__half>(pl, a_map, b_map, a, stream);
}

}  // namespace gemm
}  // namespace pdllm
