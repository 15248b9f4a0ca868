// Block-table scheduled attention over the KV cache (Flash-Cache) and the
// Flash-Verify attention, as one warp-specialised tcgen05 kernel template
// (attn_tc_kernel), plus the planner that turns the reference's block tables
// into work items and the fixed-order reduction of the attention-importance
// scores.
//
// Work item = up to 64 query rows of one sequence x one head x one slice of
// that sequence's keys.  For Flash-Cache an item holds the sequence's masked
// rows first and then its tracked (refresh) rows, so masked and tracked rows
// share one pass over K/V (the reference runs two kernels, two passes).  The
// kernel's structure is described above attn_tc_kernel.
//
// Keys of a sequence live either in its contiguous cache region
// [seq * seqlen_max, seq * seqlen_max + k_end) (the reference's layout) or,
// with a page table, in 64-row pages: key n of sequence b is cache row
// pages[b * pages_per_seq + n / 64] * 64 + n % 64.  A 64-key tile is one page,
// so either way a tile is one pair of TMA boxes.
//
// attn_scores: every (item, head) CTA adds the raw-logit column sums of its
// masked rows to a per-sequence accumulator in 2^-32 fixed point (64-bit
// integer atomics: integer addition does not depend on the order, so the sums
// -- and every refresh decision taken from them -- are the same on every
// run); the CTA that arrives last for a sequence converts its accumulator
// once into attn_scores and leaves it zeroed for the next call.
#include <cstring>

#include "common.cuh"
#include "internal.h"

namespace fdllm {

constexpr int kHD = 128;
constexpr int kItemRows = 64;
constexpr int kKeyTile = 64;
constexpr int kHalfBytes = kKeyTile * 128;          // 64 rows x 128 B (64 dims)
constexpr int kTileBytes = 2 * kHalfBytes;          // one K or V tile (128 dims)
// Plan layout (int32): header, then `capacity` items of kPlanItem, then
// kPlanSeq ints per sequence.
//   header:   [0] items, [1] batch, [2] items holding masked rows ("masked
//             items", numbered in item order), [3] offset of the per-sequence
//             section
//   item:     [0] seq, [1] k_end, [2] masked row start, [3] masked rows,
//             [4] tracked row start, [5] tracked rows, [6] masked-item number
//             (-1: no masked rows), [7] 0
//   sequence: [0] number of its first masked item, [1] its masked items
//             (consecutive), [2] k_end (0: no rows)
constexpr int kPlanHeader = 8;
constexpr int kPlanItem = 8;
constexpr int kPlanSeq = 3;
constexpr int kAttnKernelId = 2;
constexpr int kPlanKernelId = 3;

// Byte offset of 16-byte chunk `chunk` (0..15, 8 dims each) of key row `row`
// inside a tile stored as two 64-dim halves with the 128-byte swizzle -- the
// layout a SWIZZLE_128B TMA box of {64 dims, 64 rows} produces.
__device__ __forceinline__ uint32_t tile_off(int row, int chunk) {
  return (chunk >> 3) * kHalfBytes + row * 128 + (((chunk & 7) ^ (row & 7)) << 4);
}

// 16-byte async copy; with valid == false nothing is read and 16 zero bytes land.
__device__ __forceinline__ void cp_async_16_zfill(void* smem_dst, const void* gmem_src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src),
               "r"(valid ? 16 : 0)
               : "memory");
}

struct AttnParams {
  const __nv_bfloat16* q;
  __nv_bfloat16* o;
  const __nv_bfloat16* kc;      // cache K
  const __nv_bfloat16* vc;      // cache V
  const __nv_bfloat16* k1;      // verify: fresh K/V of the verify rows (row-indexed)
  const __nv_bfloat16* v1;
  const int32_t* plan;          // cache mode: plan from fdllm_plan_cache_attention
  const int32_t* vblocks;       // verify mode: (k_s, k_e, q_s, q_e) rows
  const int64_t* pos_k;         // verify mode: gathered key slots
  const uint8_t* mask;          // verify mode: [n_blocks*block_rows, block_rows]
  unsigned long long* score_acc;  // cache mode with scores: [batch][seqlen_max] fixed-point column sums
  int32_t* score_cnt;           // cache mode with scores: [batch] arrivals
  float* scores;                // cache mode: attn_scores (NULL: none)
  const int32_t* pages;         // cache mode, optional: page table [batch][pages_per_seq]
  int32_t* status;
  int64_t n_slots;
  int64_t n_pos_k;
  float scale_log2;             // softmax_scale * log2(e)
  float score_scale;
  int32_t d_model;
  int32_t n_heads;
  int32_t seqlen_max;
  int32_t kv_splits;
  int32_t n_items;              // verify mode: n_blocks * row chunks
  int32_t max_items;            // cache mode: plan entries (capacity) the launch covers
  int32_t block_rows;           // verify mode
  int32_t row_chunks;           // verify mode: ceil(block_rows / 64)
  int32_t n_rows;               // rows of q / o (and of k1 / v1 in verify mode)
  int32_t pages_per_seq;        // cache mode with a page table
};

// Item description resolved by every thread of the CTA.
struct Item {
  int seq;          // cache mode: sequence slot; verify mode: verify block index
  int n_keys;       // keys of the cache part (contiguous range or gathered list)
  int k_base;       // verify: offset into pos_k
  int rows;         // query rows in this item (<= 64)
  int m_start, m_len, t_start;   // row segments: [m_start, +m_len) then [t_start, ...)
  int blk_rows;     // verify: rows of the block, also its in-block key count
  int blk_q0;       // verify: first row of the block (q_s)
  int chunk_row0;   // verify: first block row of this item (64 * chunk)
  int mchunk;       // cache: masked-item number of the item (-1: no masked rows)
};

__device__ __forceinline__ int item_row(const Item& it, int r) {
  return r < it.m_len ? it.m_start + r : it.t_start + (r - it.m_len);
}

__device__ __forceinline__ bool load_item(const AttnParams& p, bool verify, int item_id, Item& it) {
  if (!verify) {
    // the entry (inside the plan's capacity) and the item count are read
    // together, then the entry is used only below the count
    if (item_id >= p.max_items) return false;
    const int4* e = reinterpret_cast<const int4*>(p.plan + kPlanHeader + item_id * kPlanItem);
    const int n_items = p.plan[0];
    const int4 e0 = e[0], e1 = e[1];
    if (item_id >= n_items) return false;
    it.seq = e0.x;
    it.n_keys = e0.y;
    it.m_start = e0.z;
    it.m_len = e0.w;
    it.t_start = e1.x;
    it.rows = e0.w + e1.y;
    it.mchunk = e1.z;
    return it.rows > 0;
  }
  if (item_id >= p.n_items) return false;
  const int b = item_id / p.row_chunks;
  const int c = item_id % p.row_chunks;
  const int32_t* r = p.vblocks + 4 * b;
  const int k_s = r[0], k_e = r[1], q_s = r[2];
  const int q_e = min(r[3], p.n_rows);  // rows past the query tensors are never read
  if (q_s < 0 || r[3] > p.n_rows || k_s < 0) {
    if (c == 0) report(p.status, FDLLM_ERR_TABLE, b, kAttnKernelId);
    return false;
  }
  it.seq = b;
  it.k_base = k_s;
  it.n_keys = max(0, k_e - k_s);
  it.blk_q0 = q_s;
  it.blk_rows = max(0, min(q_e - q_s, p.block_rows));
  it.chunk_row0 = c * kItemRows;
  it.m_start = q_s + c * kItemRows;
  it.m_len = max(0, min(kItemRows, it.blk_rows - c * kItemRows));
  it.t_start = 0;
  it.rows = it.m_len;
  return it.rows > 0;
}

// ---------------------------------------------------------------------------
// tcgen05 attention (Flash-Cache and Flash-Verify).  The products run on the
// 5th-generation tensor cores: S = Q K^T and O += P V are
// M=128 UMMAs issued by one thread, S (double-buffered) and the O accumulator
// live in tensor memory, and only P passes through shared memory (bf16,
// 128-byte swizzled: the A operand of the second product).  V is read in
// place as an MN-major B operand.  Cache items stream contiguous K/V ranges
// with TMA; verify items gather theirs with cp.async (the pos_k list, then
// the block's own k1 / v1 rows under the verify mask).
//
// A kernel that uses tensor memory runs one CTA per SM, so each CTA runs two
// independent pipelines ("halves"), each on its own work item -- items 2x and
// 2x+1 for grid index x / kv_splits -- with its own shared memory, barriers
// and 256 TMEM columns.  With kv_splits = S > 1 (S in {2, 4, 8}) the S CTAs
// x = kv_splits * pair + s form a cluster, CTA s taking key slice s of both
// items; each CTA leaves its unnormalised O rows and (m, l) in its own shared
// memory and, after a cluster barrier, merges rows [64 s / S, 64 (s+1) / S)
// of both items from all S CTAs through distributed shared memory.  A tcgen05.mma costs about the same issue time for any
// M <= 128 and N <= 128, so each half issues few, wide ones: per 64-key tile
// one M=128, N=64 S product (8 K-steps) and one M=128, N=128 PV product
// (4 K-steps).  The 128 rows of a half's S operand are its 64 query rows and
// qbar = the fp32 sum of its masked query rows split into bf16 hi + lo, whose
// S rows are exactly the raw-logit column sums the reference accumulates into
// attn_scores -- computed by the same instruction.  Half 0 keeps its query
// rows in rows / TMEM lanes 0-63 and qbar in 64-65; half 1 the other way
// round (qbar 0-1, query rows 64-127), so the two halves' softmax warps sit in
// different TMEM lane quarters, i.e. on different SM sub-partitions.  Operand
// rows that carry nothing are never read back, so their shared-memory windows
// may overlap other buffers.
//
// Warps (12): softmax h0: 0,1 (lanes 0-63)   softmax h1: 2,3 (lanes 64-127)
//             scores  h1: 4 (lanes 0-31)     scores  h0: 6 (lanes 64-95)
//             MMA h0: 5, h1: 7     K producer h0: 8, h1: 10     V producer
//             h0: 9, h1: 11.  Warp 8 owns TMEM (512 columns).
// Softmax: thread = one query row, all 64 keys of a tile.  The reference max
// of a row only moves (and O is rescaled in TMEM) when a tile raises the row
// max by more than 2^8, so P stays within bf16 range and O is rarely touched;
// l and O always share the reference max.
// Per 64-key tile t of a half (3 K and 2 V stages, 2 S buffers, 1 P buffer):
//   producers: K(t) -> k_full, V(t) -> v_full (never waiting on each other)
//   MMA:       S(t) -> s_full, k_empty;  then PV(t-1) after p_full(t-1) ->
//              pv_done, v_empty
//   softmax:   S(t) -> s_empty;  P(t) -> p_full once PV(t-1) freed the buffer
//   scores:    S(t) rows of qbar -> s_empty, column sums to the workspace
// K(t+3) can only be requested once S(t) is done, and S(t+3) must be done
// when the softmax reaches tile t+3, so a tile period has to cover a third of
// (K load latency + S product); with two K stages it was half of it, which
// set the period (1.15 us per tile measured at full load, against 0.8 us of
// softmax).  The third K stage is paid for with the second P buffer, which
// bought little: the softmax of tile t computes its exponentials before it
// needs PV(t-1) done.  V has slack: V(t+2) is requested when PV(t) is done
// and needed a whole softmax period after PV(t+1).
// ---------------------------------------------------------------------------
constexpr int kTcWarps = 12;
constexpr int kTcThreads = kTcWarps * 32;
constexpr uint32_t kTcTmemCols = 512;
constexpr float kTcRescaleThreshold = 8.f;  // log2 units
constexpr int kTcPBytes = kItemRows * 128;  // 64 rows x 64 keys
constexpr int kTcWin = 128 * 128;           // bytes an M=128 A operand reads from its base
constexpr int kKStages = 3;
constexpr int kVStages = 2;
// Half 0 (query rows 0-63, qbar rows 64/65): Q halves of 72 rows (9 KB) each,
// one P buffer, the K and V stages.
constexpr int kH0Q0 = 0, kH0Q1 = 9 * 1024, kH0P = 18 * 1024, kH0K = 26 * 1024,
              kH0V = kH0K + kKStages * kTileBytes, kH0End = kH0V + kVStages * kTileBytes;
// Half 1 (qbar rows 0/1, query rows 64-127): Q windows of 16 KB each, the
// query rows in their second 8 KB; the P buffer is read from 8 KB before it.
// Both halves' score scratch and barriers sit in rows 8-23 of half 1's first
// Q window, which carry nothing (only its rows 0-7 and 64-127 hold data).
constexpr int kH1Base = kH0End;
constexpr int kH1Q0 = kH1Base, kH1Scr = kH1Base + 1024, kH1Bar = kH1Scr + 512, kH0Scr = kH1Base + 2 * 1024,
              kH0Bar = kH0Scr + 512, kH1Q1 = kH1Base + 16 * 1024, kH1P = kH1Base + 32 * 1024,
              kH1K = kH1Base + 40 * 1024, kH1V = kH1K + kKStages * kTileBytes,
              kH1End = kH1V + kVStages * kTileBytes;
constexpr int kTcSmem = 1024 + kH1End;  // + alignment of the base to 1024 bytes
static_assert(kH0Q0 + kTcWin <= kH1End && kH0Q1 + kTcWin <= kH1End && kH0P + kTcWin <= kH1End,
              "half-0 operand windows inside shared memory");
static_assert(kH1P - 8 * 1024 >= kH1Q1 && kH1P + kTcPBytes <= kH1K && kH1Q1 + kTcWin <= kH1End,
              "half-1 operand windows inside shared memory");
static_assert(kH0P + kTcPBytes <= kH0K && kH1Scr >= kH1Q0 + 1024 && kH1Bar + 512 <= kH0Scr &&
                  kH0Bar + 512 <= kH1Q0 + 8 * 1024,
              "scratch and barriers outside the data rows");
static_assert(kTcSmem <= 227 * 1024, "shared memory");
static_assert(kKStages * kTileBytes >= kItemRows * kHD * 4, "a key slice's fp32 O rows fit the K stages");

struct TcHalf {
  uint32_t row_lane;   // TMEM lane / operand row of query row 0
  uint32_t qbar_lane;  // TMEM lane / operand row of qbar hi
  uint8_t* q_win0;     // S operand windows (64-dim halves)
  uint8_t* q_win1;
  uint8_t* p_row0;     // P buffer: address of query row 0's P row
  uint8_t* p_win;      // P buffer operand window
  uint8_t* k;          // K stage 0 (+ s * kTileBytes)
  uint8_t* v;          // V stage 0 (+ s * kTileBytes)
  float* scr;
  uint64_t* bar;
  uint32_t col;        // first TMEM column of this half
};

__device__ __forceinline__ TcHalf tc_half(uint8_t* smem, int h) {
  TcHalf H;
  H.row_lane = h ? 64u : 0u;
  H.qbar_lane = h ? 0u : 64u;
  H.q_win0 = smem + (h ? kH1Q0 : kH0Q0);
  H.q_win1 = smem + (h ? kH1Q1 : kH0Q1);
  H.p_row0 = smem + (h ? kH1P : kH0P);
  H.p_win = H.p_row0 - (h ? 8 * 1024 : 0);
  H.k = smem + (h ? kH1K : kH0K);
  H.v = smem + (h ? kH1V : kH0V);
  H.scr = reinterpret_cast<float*>(smem + (h ? kH1Scr : kH0Scr));
  H.bar = reinterpret_cast<uint64_t*>(smem + (h ? kH1Bar : kH0Bar));
  H.col = h ? 256u : 0u;
  return H;
}

// operand row `row` (0..127) of a K-major SW128 window: 16-byte chunk c
__device__ __forceinline__ uint8_t* win_chunk(uint8_t* win, int row, int c) {
  return win + row * 128 + (((c & 7) ^ (row & 7)) << 4);
}

// Rows [64 s / S, 64 (s+1) / S) of one item, merged from the key slices of
// the S CTAs of the cluster (CTA c's O rows at H.k, (m, l) at H.v, in its own
// shared memory): O = sum_c 2^(m_c - m) O_c / sum_c 2^(m_c - m) l_c.  Thread
// t of the half's 64 takes row 64 s / S + t / S and columns
// (t % S) * 128 / S ... + 128 / S.
template <int S>
__device__ __forceinline__ void tc_merge_rows(const AttnParams& p, const TcHalf& H, const Item& it, int head,
                                              int s, int t) {
  constexpr int kCols = kHD / S;  // columns per thread
  const int row = s * (kItemRows / S) + t / S;
  const int part = t % S;
  float m[S], w[S];
  float mmax = -INFINITY;
#pragma unroll
  for (int c = 0; c < S; ++c) {
    const float2 ml = ld_dsmem_f2(mapa_shared(reinterpret_cast<const float2*>(H.v) + row, c));
    m[c] = ml.x;
    w[c] = ml.y;
    mmax = fmaxf(mmax, ml.x);
  }
  const float ref = mmax == -INFINITY ? 0.f : mmax;
  float lsum = 0.f;
#pragma unroll
  for (int c = 0; c < S; ++c) {
    const float e = exp2f(m[c] - ref);
    lsum += e * w[c];
    w[c] = e;
  }
  const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
  float acc[kCols];
#pragma unroll
  for (int j = 0; j < kCols; ++j) acc[j] = 0.f;
  const uint8_t* orow = H.k + row * (kHD * 4);
#pragma unroll
  for (int c = 0; c < S; ++c) {
#pragma unroll
    for (int j = 0; j < kCols / 4; ++j) {
      const int u = part * (kCols / 4) + j;
      const float4 v = ld_dsmem_f4(mapa_shared(orow + ((u ^ (row & 7)) << 4), c));
      acc[4 * j] += w[c] * v.x;
      acc[4 * j + 1] += w[c] * v.y;
      acc[4 * j + 2] += w[c] * v.z;
      acc[4 * j + 3] += w[c] * v.w;
    }
  }
  if (row >= it.rows) return;
  __nv_bfloat16* dst = p.o + item_row(it, row) * p.d_model + head * kHD + part * kCols;
#pragma unroll
  for (int j = 0; j < kCols; j += 8) {
    uint4 v;
    v.x = pack_bf16x2(acc[j] * inv, acc[j + 1] * inv);
    v.y = pack_bf16x2(acc[j + 2] * inv, acc[j + 3] * inv);
    v.z = pack_bf16x2(acc[j + 4] * inv, acc[j + 5] * inv);
    v.w = pack_bf16x2(acc[j + 6] * inv, acc[j + 7] * inv);
    *reinterpret_cast<uint4*>(dst + j) = v;
  }
}

template <bool kVerify>
__global__ void __launch_bounds__(kTcThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap map_k, const __grid_constant__ CUtensorMap map_v,
                   const __grid_constant__ CUtensorMap map_k1, const __grid_constant__ CUtensorMap map_v1,
                   const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int head = blockIdx.y;
  // Q, the K/V rows and the plan come from the kernels before (programmatic
  // launch: this CTA may already be resident while the QKV GEMM finishes)
  pdl_wait();

  // warp -> (half, role): 0,1 softmax h0 | 2,3 softmax h1 | 4 scores h1 |
  // 5 MMA h0 | 6 scores h0 | 7 MMA h1 | 8 K h0 | 9 V h0 | 10 K h1 | 11 V h1
  enum Role { kSoftmax, kScores, kMma, kProdK, kProdV };
  const int role = warp < 4 ? kSoftmax
                   : warp >= 8 ? ((warp & 1) ? kProdV : kProdK)
                               : ((warp & 1) ? kMma : kScores);
  const int h = warp < 4 ? (warp >> 1) : warp >= 8 ? ((warp >> 1) & 1) : (warp == 4 || warp == 7) ? 1 : 0;
  const TcHalf H = tc_half(smem, h);
  uint64_t* k_full = H.bar;                                // [kKStages]
  uint64_t* k_empty = k_full + kKStages;                   // [kKStages]
  uint64_t* v_full = k_empty + kKStages;                   // [kVStages]
  uint64_t* v_empty = v_full + kVStages;                   // [kVStages]
  uint64_t* s_full = v_empty + kVStages;                   // [2]
  uint64_t* s_empty = s_full + 2;                          // [2]
  uint64_t* p_full = s_empty + 2;
  uint64_t* pv_done = p_full + 1;
  uint64_t* mma_done = pv_done + 1;
  static_assert(2 * (kKStages + kVStages) + 7 <= 17, "barriers below the fail flag");
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kH0Bar + 18 * 8);
  volatile int32_t* fail = reinterpret_cast<volatile int32_t*>(H.bar + 17);
  // sequence whose scores this half's scores warp found complete (-1: none);
  // the whole CTA converts them at the end
  volatile int32_t* convert_seq = reinterpret_cast<volatile int32_t*>(H.bar + 19);

  // this half's work item and key split (split = rank in the cluster)
  const int pair = blockIdx.x / p.kv_splits;
  const int split = blockIdx.x % p.kv_splits;
  const int item_id = 2 * pair + h;
  Item it{};
  const bool has_item = load_item(p, kVerify, item_id, it);
  // keys of this split: equal 64-aligned slices of the item's cache keys;
  // verify items add their block's own keys (last split) as further tiles
  int c0 = 0, c1 = 0, nt_cache = 0, n_tiles = 0;
  if (has_item) {
    const int per = ((it.n_keys + p.kv_splits - 1) / p.kv_splits + kKeyTile - 1) / kKeyTile * kKeyTile;
    c0 = min(it.n_keys, split * per);
    c1 = min(it.n_keys, c0 + per);
    nt_cache = (c1 - c0 + kKeyTile - 1) / kKeyTile;
    const int nt_blk = (kVerify && split == p.kv_splits - 1) ? (it.blk_rows + kKeyTile - 1) / kKeyTile : 0;
    n_tiles = nt_cache + nt_blk;
  }
  const bool scores_on = !kVerify && has_item && p.scores != nullptr && it.m_len > 0 && it.mchunk >= 0;
  const int64_t d = p.d_model;
  {
    // the CTA exits only when neither half has an item
    Item other{};
    const bool other_has = load_item(p, kVerify, 2 * pair + (1 - h), other);
    if (!has_item && !other_has) return;  // uniform across the CTA and its cluster
  }

  if (role == kMma && lane == 0) {
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], scores_on ? 3 : 2);
    }
    mbar_init(p_full, 2);
    mbar_init(pv_done, 1);
    mbar_init(mma_done, 1);
    *fail = 0;
    *convert_seq = -1;
    fence_barrier_init();
  }
  if (warp == 8) {
    tmem_alloc(tmem_slot, kTcTmemCols);
    if (lane == 0) {
      tma_prefetch_desc(&map_k);
      tma_prefetch_desc(&map_v);
      if (kVerify) {
        tma_prefetch_desc(&map_k1);
        tma_prefetch_desc(&map_v1);
      }
    }
  }
  // barriers and TMEM are ready: the producers start loading K/V at once,
  // while warps 0-7 fill the Q operands
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp < 8) {
    // operand fill of half f by threads [128 f, 128 f + 128): query rows (rows
    // past the item zero), qbar hi / lo, the other rows of qbar's 8-row atom
    // zero.  All eight loads of a thread are in flight together.
    const int f = threadIdx.x >> 7, tid = threadIdx.x & 127;
    const TcHalf F = tc_half(smem, f);
    Item fi{};
    const bool f_has = load_item(p, kVerify, 2 * pair + f, fi);
    constexpr int kPer = kItemRows * 16 / 128;
    uint4 v[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int row = (tid + 128 * k) >> 4, c = tid & 15;
      v[k] = (f_has && row < fi.rows)
                 ? *reinterpret_cast<const uint4*>(p.q + item_row(fi, row) * d + head * kHD + c * 8)
                 : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int row = (tid + 128 * k) >> 4, c = tid & 15;
      *reinterpret_cast<uint4*>(win_chunk((c >> 3) ? F.q_win1 : F.q_win0, F.row_lane + row, c)) = v[k];
    }
    if (tid < 2 * 8 * 8) {  // qbar's atom: 8 rows x 8 chunks x 2 halves
      const int hh = tid >> 6, rr = F.qbar_lane + ((tid >> 3) & 7), ch = tid & 7;
      *reinterpret_cast<uint4*>(win_chunk(hh ? F.q_win1 : F.q_win0, rr, ch)) = make_uint4(0, 0, 0, 0);
    }
    const bool f_scores = !kVerify && f_has && p.scores != nullptr && fi.m_len > 0 && fi.mchunk >= 0;
    if (f_scores) {
      // qbar = fp32 sum of the masked rows (the item's first m_len rows) ->
      // bf16 hi (row qbar_lane) and lo (row qbar_lane + 1).  Every thread
      // adds its own loaded rows (8 dims of chunk tid & 15), lanes 16 apart
      // combine, then the four warps' partials are added in warp order
      // through the P buffer (unused until the first softmax): a fixed order.
      float part[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) part[e] = 0.f;
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        if ((tid >> 4) + 8 * k < fi.m_len) {
          const __nv_bfloat162* pv = reinterpret_cast<const __nv_bfloat162*>(&v[k]);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 x = __bfloat1622float2(pv[e]);
            part[2 * e] += x.x;
            part[2 * e + 1] += x.y;
          }
        }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) part[e] += __shfl_xor_sync(0xffffffffu, part[e], 16);
      float* red = reinterpret_cast<float*>(F.p_row0);  // [4 warps][128 dims]
      if ((tid & 31) < 16) {
#pragma unroll
        for (int e = 0; e < 8; ++e) red[(tid >> 5) * kHD + (tid & 15) * 8 + e] = part[e];
      }
      if (f == 0)
        asm volatile("bar.sync 1, 128;" ::: "memory");
      else
        asm volatile("bar.sync 2, 128;" ::: "memory");
      const int dim = tid, c = (dim & 63) >> 3;
      uint8_t* win = (dim >> 6) ? F.q_win1 : F.q_win0;
      const float acc = ((red[dim] + red[kHD + dim]) + red[2 * kHD + dim]) + red[3 * kHD + dim];
      const __nv_bfloat16 hi = __float2bfloat16_rn(acc);
      const __nv_bfloat16 lo = __float2bfloat16_rn(acc - __bfloat162float(hi));
      *reinterpret_cast<__nv_bfloat16*>(win_chunk(win, F.qbar_lane, c) + (dim & 7) * 2) = hi;
      *reinterpret_cast<__nv_bfloat16*>(win_chunk(win, F.qbar_lane + 1, c) + (dim & 7) * 2) = lo;
    }
    fence_proxy_async_smem();
    asm volatile("bar.sync 3, 256;" ::: "memory");  // warps 0-7: Q in place for the S products
  }
  const uint32_t tmem = *tmem_slot + H.col;

  if ((role == kProdK || role == kProdV) && !kVerify) {
    // ------------------------------------------------- TMA producers ----
    if (lane == 0) {
      const bool is_k = role == kProdK;
      uint64_t* full = is_k ? k_full : v_full;
      uint64_t* empty = is_k ? k_empty : v_empty;
      const CUtensorMap* map = is_k ? &map_k : &map_v;
      const int n_st = is_k ? kKStages : kVStages;
      for (int t = 0; t < n_tiles; ++t) {
        const int s = t % n_st;
        if (t >= n_st && !mbar_wait(&empty[s], ((t - n_st) / n_st) & 1, p.status, kAttnKernelId)) {
          *fail = 1;
          break;
        }
        const int n0 = c0 + t * kKeyTile;  // a multiple of 64: one page
        int64_t y = static_cast<int64_t>(it.seq) * p.seqlen_max + n0;
        if (p.pages != nullptr) {
          const int64_t page = p.pages[static_cast<int64_t>(it.seq) * p.pages_per_seq + n0 / kKeyTile];
          if (page < 0 || (page + 1) * kKeyTile > p.n_slots) {
            // a page outside the cache: recorded; the tile is read from row 0
            // (in bounds) so the pipeline still completes
            if (is_k) report(p.status, FDLLM_ERR_INDEX, static_cast<int>(page), kAttnKernelId);
            y = 0;
          } else {
            y = page * kKeyTile;
          }
        }
        uint8_t* dst = (is_k ? H.k : H.v) + s * kTileBytes;
        mbar_arrive_expect_tx(&full[s], kTileBytes);
        tma_load_2d(dst, map, head * kHD, static_cast<int32_t>(y), &full[s]);
        tma_load_2d(dst + kHalfBytes, map, head * kHD + 64, static_cast<int32_t>(y), &full[s]);
      }
    }
  } else if (role == kProdK || role == kProdV) {
    // ---------------------------------------------- gather producers ----
    // Verify keys: cache rows listed in pos_k, then the block's own rows of
    // k1 / v1.  A tile whose 64 keys are 64 consecutive rows (the common case:
    // the key list is a few runs of cache slots) is one pair of TMA boxes;
    // any other tile is gathered with 16-byte cp.async per lane, zero-filled
    // for missing keys, and published once the copies of the next gathered
    // tile are in flight.
    const bool is_k = role == kProdK;
    uint64_t* full = is_k ? k_full : v_full;
    uint64_t* empty = is_k ? k_empty : v_empty;
    const int n_st = is_k ? kKStages : kVStages;
    bool ok = true;
    int pending = -1;  // stage of the gathered tile not yet published
    int s = n_st - 1, use = -1;  // stage of tile t, and how often it was filled before
    for (int t = 0; t < n_tiles; ++t) {
      if (++s == n_st) {
        s = 0;
        ++use;
      }
      // the tile's key rows are read before waiting for its stage, so the
      // position loads overlap the wait
      const bool blk = t >= nt_cache;
      const int n0 = blk ? (t - nt_cache) * kKeyTile : c0 + t * kKeyTile;
      const int n_end = blk ? it.blk_rows : c1;
      int64_t src_row[2];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int n = n0 + lane + 32 * hh;
        int64_t row = -1;
        if (n < n_end) {
          if (blk) {
            row = it.blk_q0 + n;
          } else {
            const int64_t pk = static_cast<int64_t>(it.k_base) + n;
            row = (pk < p.n_pos_k) ? p.pos_k[pk] : -1;
          }
        }
        src_row[hh] = row;
      }
      if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1, p.status, kAttnKernelId)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int n = n0 + lane + 32 * hh;
        if (!blk && n < n_end && (src_row[hh] < 0 || src_row[hh] >= p.n_slots)) {
          if (is_k) report(p.status, FDLLM_ERR_INDEX, static_cast<int>(it.k_base + n), kAttnKernelId);
          src_row[hh] = -1;
        }
      }
      uint8_t* dst = (is_k ? H.k : H.v) + s * kTileBytes;
      const int64_t row0 = __shfl_sync(0xffffffffu, src_row[0], 0);
      const bool run = __all_sync(0xffffffffu, row0 >= 0 && src_row[0] == row0 + lane && src_row[1] == row0 + lane + 32);
      if (run) {
        // publish the gathered tile before it, then load this one with TMA
        if (pending >= 0) {
          asm volatile("cp.async.wait_group 0;" ::: "memory");
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&full[pending]);
          pending = -1;
        }
        if (lane == 0) {
          const CUtensorMap* map = is_k ? (blk ? &map_k1 : &map_k) : (blk ? &map_v1 : &map_v);
          mbar_arrive_expect_tx(&full[s], kTileBytes);
          tma_load_2d(dst, map, head * kHD, static_cast<int32_t>(row0), &full[s]);
          tma_load_2d(dst + kHalfBytes, map, head * kHD + 64, static_cast<int32_t>(row0), &full[s]);
        }
        continue;
      }
      const __nv_bfloat16* src = is_k ? (blk ? p.k1 : p.kc) : (blk ? p.v1 : p.vc);
#pragma unroll 8
      for (int i = 0; i < kKeyTile / 2; ++i) {
        const int key = 2 * i + (lane >> 4);
        const int chunk = lane & 15;
        const int64_t r0 = __shfl_sync(0xffffffffu, src_row[0], key & 31);
        const int64_t r1 = __shfl_sync(0xffffffffu, src_row[1], key & 31);
        const int64_t row = key < 32 ? r0 : r1;
        const bool valid = row >= 0;
        cp_async_16_zfill(dst + tile_off(key, chunk), src + (valid ? row * d + head * kHD + chunk * 8 : 0), valid);
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
      if (pending >= 0) {
        asm volatile("cp.async.wait_group 1;" ::: "memory");
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full[pending]);
      }
      pending = s;
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    fence_proxy_async_smem();
    __syncwarp();
    if (ok && pending >= 0 && lane == 0) mbar_arrive(&full[pending]);
    if (!ok) *fail = 1;
  } else if (role == kMma) {
    // ------------------------------------------------------------ MMA ----
    if (lane == 0) {
      const uint32_t idesc_s = umma_idesc_bf16(128, kKeyTile);
      const uint32_t idesc_pv = umma_idesc_bf16(128, kHD) | kUmmaBMajorMN;
      // descriptors of the operand bases; +16 B adds 1 to the start field
      const uint64_t dq0 = umma_desc_kmajor_sw128(smem_u32(H.q_win0));
      const uint64_t dq1 = umma_desc_kmajor_sw128(smem_u32(H.q_win1));
      const uint64_t pa = umma_desc_kmajor_sw128(smem_u32(H.p_win));
      auto pv = [&](int u) -> bool {
        const int vs = u % kVStages;
        if (!mbar_wait(p_full, u & 1, p.status, kAttnKernelId)) return false;
        if (!mbar_wait(&v_full[vs], (u / kVStages) & 1, p.status, kAttnKernelId)) return false;
        tc_fence_after();
        const uint64_t va = umma_desc_mnmajor_sw128(smem_u32(H.v + vs * kTileBytes), kHalfBytes);
#pragma unroll
        for (int kk = 0; kk < kKeyTile / 16; ++kk)
          umma_bf16(tmem + 128, pa + (kk * 32 >> 4), va + (kk * 2048 >> 4), idesc_pv, (u > 0 || kk > 0) ? 1u : 0u);
        umma_commit(pv_done);
        umma_commit(&v_empty[vs]);
        return true;
      };
      bool ok = true;
      for (int t = 0; t < n_tiles && ok; ++t) {
        const int s = t & 1;  // S buffer
        const int ks = t % kKStages;
        ok = mbar_wait(&k_full[ks], (t / kKStages) & 1, p.status, kAttnKernelId) &&
             (t < 2 || mbar_wait(&s_empty[s], ((t - 2) >> 1) & 1, p.status, kAttnKernelId));
        if (!ok) break;
        tc_fence_after();
        const uint64_t ka = umma_desc_kmajor_sw128(smem_u32(H.k + ks * kTileBytes));
#pragma unroll
        for (int kk = 0; kk < kHD / 16; ++kk)
          umma_bf16(tmem + kKeyTile * s, ((kk >> 2) ? dq1 : dq0) + ((kk & 3) * 32 >> 4),
                    ka + (((kk >> 2) * kHalfBytes + (kk & 3) * 32) >> 4), idesc_s, kk > 0 ? 1u : 0u);
        umma_commit(&s_full[s]);
        umma_commit(&k_empty[ks]);
        if (t >= 1) ok = pv(t - 1);
      }
      if (ok && n_tiles > 0) ok = pv(n_tiles - 1);
      if (!ok) *fail = 1;
      // every issued MMA has completed before TMEM can be released
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, p.status, kAttnKernelId);
    }
  } else if (role == kScores) {
    // ------------------------------------------------------- scores ----
    if (scores_on) {
      // S rows qbar (hi) and qbar + 1 (lo) are this warp's lanes 0 and 1:
      // they stage the 64 column values of a tile, every lane then adds hi +
      // lo of two columns to the sequence's fixed-point accumulator
      unsigned long long* acc = p.score_acc + static_cast<int64_t>(it.seq) * p.seqlen_max;
      const uint32_t taddr = tmem + (H.qbar_lane << 16);
      bool range_ok = true;
      for (int t = 0; t < n_tiles; ++t) {
        const int b = t & 1;
        if (!mbar_wait(&s_full[b], (t >> 1) & 1, p.status, kAttnKernelId)) {
          *fail = 1;
          break;
        }
        tc_fence_after();
        float sc[64];
        tmem_ld_32x32b_x32(taddr + kKeyTile * b, *reinterpret_cast<float(*)[32]>(&sc[0]));
        tmem_ld_32x32b_x32(taddr + kKeyTile * b + 32, *reinterpret_cast<float(*)[32]>(&sc[32]));
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_empty[b]);
        if (lane < 2) {
#pragma unroll
          for (int j = 0; j < 64; j += 4)
            *reinterpret_cast<float4*>(H.scr + 64 * lane + j) = make_float4(sc[j], sc[j + 1], sc[j + 2], sc[j + 3]);
        }
        __syncwarp();
        const int n0 = c0 + t * kKeyTile;
        const int n_valid = c1 - n0;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int j = lane + 32 * hh;
          if (j < n_valid) {
            const float x = H.scr[j] + H.scr[64 + j];
            // |x| < 2^24: x * 2^32 is exact in fp32 and up to 128 such terms
            // per key stay inside int64
            const bool in_range = fabsf(x) < 16777216.f;  // false for NaN / inf
            range_ok &= in_range;
            atomicAdd(acc + n0 + j,
                      static_cast<unsigned long long>(in_range ? __float2ll_rn(x * 4294967296.f) : 0ll));
          }
        }
        __syncwarp();
      }
      if (!__all_sync(0xffffffffu, range_ok) && lane == 0) report(p.status, FDLLM_ERR_RANGE, it.seq, kAttnKernelId);
      // arrival: the last (item, head, split) of the sequence to arrive hands
      // it to its CTA for conversion at the end
      __threadfence();
      __syncwarp();
      if (lane == 0) {
        const int expected = p.plan[p.plan[3] + kPlanSeq * it.seq + 1] * p.n_heads * p.kv_splits;
        if (atomicAdd(p.score_cnt + it.seq, 1) == expected - 1) {
          p.score_cnt[it.seq] = 0;
          __threadfence();
          *convert_seq = it.seq;
        }
      }
    }
  } else {
    // ------------------------------------------------------- softmax ----
    const int r = (warp & 1) * 32 + lane;  // item row
    const bool row_ok = has_item && r < it.rows;
    const uint32_t trow = tmem + ((H.row_lane + static_cast<uint32_t>((warp & 1) * 32)) << 16);
    const uint8_t* mrow = nullptr;  // verify: this row's in-block mask
    if (kVerify && has_item) {
      const int64_t base = static_cast<int64_t>(it.seq) * p.block_rows + it.chunk_row0;
      mrow = p.mask + (base + min(r, max(it.rows - 1, 0))) * p.block_rows;
    }
    // verify: the row's first 64 in-block mask bytes, loaded while the cache
    // tiles run (the in-block tiles come last)
    uint4 mask_w[4] = {};
    const bool mask_pre = kVerify && has_item && it.blk_rows > 0 && p.block_rows % 16 == 0 &&
                          (reinterpret_cast<uintptr_t>(mrow) & 15) == 0;
    if (mask_pre) {
#pragma unroll
      for (int k = 0; k < 4; ++k)  // within this row's block_rows bytes
        if (16 * k < it.blk_rows && 16 * k + 16 <= p.block_rows)
          mask_w[k] = __ldg(reinterpret_cast<const uint4*>(mrow) + k);
    }
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int t = 0; t < n_tiles; ++t) {
      const int b = t & 1;
      ok = mbar_wait(&s_full[b], (t >> 1) & 1, p.status, kAttnKernelId);
      if (!ok) break;
      tc_fence_after();
      float sv[64];
      tmem_ld_32x32b_x32(trow + kKeyTile * b, *reinterpret_cast<float(*)[32]>(&sv[0]));
      tmem_ld_32x32b_x32(trow + kKeyTile * b + 32, *reinterpret_cast<float(*)[32]>(&sv[32]));
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[b]);

      const bool blk = kVerify && t >= nt_cache;
      const int n0 = blk ? (t - nt_cache) * kKeyTile : c0 + t * kKeyTile;
      const int n_valid = (blk ? it.blk_rows : c1) - n0;
      const bool full = n_valid >= kKeyTile;  // uniform
      if (blk && n0 == 0 && mask_pre) {
        // the block's own keys: key range and the verify mask of this row
        const uint8_t* mb = reinterpret_cast<const uint8_t*>(mask_w);
#pragma unroll
        for (int j = 0; j < 64; ++j) sv[j] = (j < n_valid && mb[j] != 0) ? sv[j] : -INFINITY;
      } else if (blk) {
#pragma unroll
        for (int j = 0; j < 64; ++j) sv[j] = (j < n_valid && __ldg(mrow + n0 + j) != 0) ? sv[j] : -INFINITY;
      } else if (!full) {
        // keys past the range: -inf logits (probability 0 below)
#pragma unroll
        for (int j = 0; j < 64; ++j) sv[j] = j < n_valid ? sv[j] : -INFINITY;
      }
      float mx[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx[i] = sv[i];
#pragma unroll
      for (int j = 8; j < 64; ++j) mx[j & 7] = fmaxf(mx[j & 7], sv[j]);
#pragma unroll
      for (int i = 4; i > 0; i >>= 1)
#pragma unroll
        for (int k = 0; k < i; ++k) mx[k] = fmaxf(mx[k], mx[k + i]);
      const float mt = mx[0] * p.scale_log2;  // scale > 0; -inf stays -inf
      const float m_new = fmaxf(m_used, mt);
      const bool need = row_ok && m_new > m_used + kTcRescaleThreshold;
      const float alpha = need ? exp2f(m_used - m_new) : 1.f;  // m_used = -inf -> 0
      // O holds PV(0..t-1): rescale it when a row of the warp moves its max
      if (__any_sync(0xffffffffu, need) && t > 0) {
        ok = mbar_wait(pv_done, (t - 1) & 1, p.status, kAttnKernelId);
        if (!ok) break;
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < kHD / 32; ++c) {
          float ov[32];
          tmem_ld_32x32b_x32(trow + 128 + 32 * c, ov);
#pragma unroll
          for (int j = 0; j < 32; ++j) ov[j] *= alpha;
          tmem_st_32x32b_x32(trow + 128 + 32 * c, ov);
        }
      }
      if (need) {
        l *= alpha;
        m_used = m_new;
      }
      const float nref = -(m_used == -INFINITY ? 0.f : m_used);
      const float scale = p.scale_log2;
      // p = 2^(s * scale - ref), masked keys 0
      float ps[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) ps[i] = 0.f;
#pragma unroll
      for (int j = 0; j < 64; ++j) {
        sv[j] = ex2_approx(fmaf(sv[j], scale, nref));  // -inf -> 0
        ps[j & 7] += sv[j];
      }
#pragma unroll
      for (int i = 4; i > 0; i >>= 1)
#pragma unroll
        for (int k = 0; k < i; ++k) ps[k] += ps[k + i];
      l += ps[0];
      // the P buffer was last read by PV(t-1)
      if (t >= 1) {
        ok = mbar_wait(pv_done, (t - 1) & 1, p.status, kAttnKernelId);
        if (!ok) break;
      }
      // (the row address is formed per tile: hoisted out of the loop, the
      // 64-bit pointer would hold two registers across it and spill)
      int zero;
      asm volatile("mov.b32 %0, 0;" : "=r"(zero));
      uint8_t* prow = H.p_row0 + zero + r * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) << 4)) =
            make_uint4(pack_bf16x2(sv[8 * c], sv[8 * c + 1]), pack_bf16x2(sv[8 * c + 2], sv[8 * c + 3]),
                       pack_bf16x2(sv[8 * c + 4], sv[8 * c + 5]), pack_bf16x2(sv[8 * c + 6], sv[8 * c + 7]));
      if (!kVerify && !full) {
        // TMA brought whole rows past the end of this key range: zero their V
        // so 0-probability keys cannot inject non-finite cache contents.
        ok = mbar_wait(&v_full[t % kVStages], (t / kVStages) & 1, p.status, kAttnKernelId);
        if (!ok) break;
        for (int idx = r; idx < (kKeyTile - n_valid) * 16; idx += 64) {
          const int key = n_valid + idx / 16, chunk = idx % 16;
          *reinterpret_cast<uint4*>(H.v + (t % kVStages) * kTileBytes + tile_off(key, chunk)) =
              make_uint4(0, 0, 0, 0);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (!ok) *fail = 1;

    // ------------------------------------------------------ epilogue ----
    const bool have_o = ok && n_tiles > 0 && mbar_wait(pv_done, (n_tiles - 1) & 1, p.status, kAttnKernelId);
    if (have_o) tc_fence_after();
    if (has_item) {
      const int64_t grow = row_ok ? item_row(it, r) : 0;
      if (p.kv_splits == 1) {
        const float inv = (have_o && l > 0.f) ? 1.f / l : 0.f;
        __nv_bfloat16* orow = p.o + grow * d + head * kHD;
#pragma unroll 1
        for (int c = 0; c < kHD / 32; ++c) {
          float ov[32];
          if (have_o) {
            tmem_ld_32x32b_x32(trow + 128 + 32 * c, ov);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) ov[j] = 0.f;
          }
          if (row_ok) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
              uint4 v;
              v.x = pack_bf16x2(ov[j] * inv, ov[j + 1] * inv);
              v.y = pack_bf16x2(ov[j + 2] * inv, ov[j + 3] * inv);
              v.z = pack_bf16x2(ov[j + 4] * inv, ov[j + 5] * inv);
              v.w = pack_bf16x2(ov[j + 6] * inv, ov[j + 7] * inv);
              *reinterpret_cast<uint4*>(orow + 32 * c + j) = v;
            }
          }
        }
      } else {
        // Key slice of a cluster: this split's unnormalised O row (fp32,
        // 16-byte units XOR-swizzled by row) goes to the half's K stages and
        // (m, l) to its V stages -- both idle once the last PV product is done
        uint8_t* orow = H.k + r * (kHD * 4);
#pragma unroll 1
        for (int c = 0; c < kHD / 32; ++c) {
          float ov[32];
          if (have_o) {
            tmem_ld_32x32b_x32(trow + 128 + 32 * c, ov);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) ov[j] = 0.f;
          }
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<float4*>(orow + (((c * 8 + j) ^ (r & 7)) << 4)) =
                make_float4(ov[4 * j], ov[4 * j + 1], ov[4 * j + 2], ov[4 * j + 3]);
        }
        reinterpret_cast<float2*>(H.v)[r] = make_float2(have_o ? m_used : -INFINITY, have_o ? l : 0.f);
      }
    }
  }

  if (p.kv_splits > 1) {
    // every thread of the cluster: the partials are in place ...
    cluster_sync_all();
    if (role == kSoftmax && has_item) {
      const int t = (warp & 1) * 32 + lane;
      if (p.kv_splits == 2)
        tc_merge_rows<2>(p, H, it, head, split, t);
      else if (p.kv_splits == 4)
        tc_merge_rows<4>(p, H, it, head, split, t);
      else
        tc_merge_rows<8>(p, H, it, head, split, t);
    }
    // ... and stay readable until every CTA of the cluster has merged
    cluster_sync_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(*tmem_slot, kTcTmemCols);
  }
  if (!kVerify && p.scores != nullptr) {
    // every (item, head, split) of a sequence handed here has added its
    // column sums (each fenced before its arrival): read the accumulator row
    // from L2, zero it, add it once to attn_scores; all threads, their loads
    // in flight together
#pragma unroll 1
    for (int hh = 0; hh < 2; ++hh) {
      const int seq = *reinterpret_cast<volatile int32_t*>(tc_half(smem, hh).bar + 19);
      if (seq < 0) continue;  // uniform
      const int k_end = min(p.plan[p.plan[3] + kPlanSeq * seq + 2], p.seqlen_max);
      unsigned long long* acc = p.score_acc + static_cast<int64_t>(seq) * p.seqlen_max;
      float* dst = p.scores + static_cast<int64_t>(seq) * p.seqlen_max;
      for (int n0 = 0; n0 < k_end; n0 += 4 * kTcThreads) {
        long long v[4];
        float old[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int n = n0 + threadIdx.x + kTcThreads * u;
          v[u] = n < k_end ? __ldcg(reinterpret_cast<const long long*>(acc + n)) : 0ll;
          old[u] = n < k_end ? dst[n] : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int n = n0 + threadIdx.x + kTcThreads * u;
          if (n < k_end) {
            __stcg(reinterpret_cast<long long*>(acc + n), 0ll);
            dst[n] = old[u] + static_cast<float>(static_cast<double>(v[u]) * 2.3283064365386963e-10) * p.score_scale;
          }
        }
      }
    }
  }
}

// ------------------------------------------------------------ planner ----
constexpr int kPlanThreads = 1024;
constexpr int kPlanMaxBatch = 1024;

__global__ void __launch_bounds__(kPlanThreads) plan_kernel(const int64_t* __restrict__ masked, int n_masked,
                                                            const int64_t* __restrict__ tracked, int n_tracked,
                                                            int batch, int block_m, int seqlen_max, int n_rows,
                                                            int capacity, int32_t* __restrict__ plan,
                                                            int32_t* status) {
  __shared__ int m_start[kPlanMaxBatch], m_len[kPlanMaxBatch], m_cnt[kPlanMaxBatch];
  __shared__ int t_min[kPlanMaxBatch], t_max[kPlanMaxBatch], t_len[kPlanMaxBatch];
  __shared__ int k_end[kPlanMaxBatch], n_it[kPlanMaxBatch], off[kPlanMaxBatch], moff[kPlanMaxBatch];
  __shared__ int bad;
  const int tid = threadIdx.x;
  if (tid == 0) bad = 0;
  for (int b = tid; b < batch; b += kPlanThreads) {
    m_start[b] = 0;
    m_len[b] = 0;
    m_cnt[b] = 0;
    t_min[b] = INT32_MAX;
    t_max[b] = -1;
    t_len[b] = 0;
    k_end[b] = -1;
  }
  __syncthreads();
  for (int i = tid; i < n_masked + n_tracked; i += kPlanThreads) {
    const bool is_m = i < n_masked;
    const int64_t* r = is_m ? masked + 4 * i : tracked + 4 * (i - n_masked);
    const int64_t b = r[0], ke = r[1], qs = r[2], qe = r[3];
    if (b < 0 || b >= batch || ke <= 0 || ke > seqlen_max || qs < 0 || qe <= qs || qe - qs > block_m ||
        qe > n_rows) {
      atomicExch(&bad, i + 1);
      continue;
    }
    const int prev = atomicCAS(&k_end[b], -1, static_cast<int>(ke));
    if (prev != -1 && prev != ke) atomicExch(&bad, i + 1);
    if (is_m) {
      if (atomicAdd(&m_cnt[b], 1) != 0) atomicExch(&bad, i + 1);
      m_start[b] = static_cast<int>(qs);
      m_len[b] = static_cast<int>(qe - qs);
    } else {
      atomicMin(&t_min[b], static_cast<int>(qs));
      atomicMax(&t_max[b], static_cast<int>(qe));
      atomicAdd(&t_len[b], static_cast<int>(qe - qs));
    }
  }
  __syncthreads();
  for (int b = tid; b < batch; b += kPlanThreads) {
    if (t_len[b] > 0 && t_max[b] - t_min[b] != t_len[b]) atomicExch(&bad, n_masked + 1);
    const int rows = m_len[b] + t_len[b];
    n_it[b] = rows > 0 ? (rows + kItemRows - 1) / kItemRows : 0;
  }
  __syncthreads();
  const int seq_off = kPlanHeader + capacity * kPlanItem;
  if (tid == 0) {
    int acc = 0, macc = 0;
    for (int b = 0; b < batch; ++b) {
      off[b] = acc;
      acc += n_it[b];
      moff[b] = macc;
      macc += (m_len[b] + kItemRows - 1) / kItemRows;
    }
    if (acc > capacity) bad = -1;
    plan[0] = bad != 0 ? 0 : acc;
    plan[1] = batch;
    plan[2] = bad != 0 ? 0 : macc;
    plan[3] = seq_off;
    if (bad != 0) report(status, FDLLM_ERR_TABLE, bad, kPlanKernelId);
  }
  __syncthreads();
  for (int b = tid; b < batch; b += kPlanThreads) {
    int32_t* e = plan + seq_off + kPlanSeq * b;
    const bool live = bad == 0 && m_len[b] + t_len[b] > 0;
    e[0] = live ? moff[b] : 0;
    e[1] = live ? (m_len[b] + kItemRows - 1) / kItemRows : 0;
    e[2] = live ? k_end[b] : 0;
  }
  if (bad != 0) return;
  for (int b = tid; b < batch; b += kPlanThreads) {
    const int rows = m_len[b] + t_len[b];
    for (int k = 0; k < n_it[b]; ++k) {
      const int v0 = k * kItemRows, v1 = min(rows, v0 + kItemRows);
      const int mseg = max(0, min(v1, m_len[b]) - v0);
      const int tfrom = max(v0, m_len[b]);
      int32_t* e = plan + kPlanHeader + (off[b] + k) * kPlanItem;
      e[0] = b;
      e[1] = k_end[b];
      e[2] = m_start[b] + v0;
      e[3] = mseg;
      e[4] = t_len[b] > 0 ? t_min[b] + (tfrom - m_len[b]) : 0;
      e[5] = max(0, v1 - tfrom);
      e[6] = mseg > 0 ? moff[b] + k : -1;
      e[7] = 0;
    }
  }
}

namespace {

int plan_capacity(int32_t n_rows, int32_t batch) { return (n_rows + kItemRows - 1) / kItemRows + batch; }

// Workspace of fdllm_attn_cache with scores: a fixed-point accumulator row
// per sequence and an arrival counter per sequence (the batch is at most the
// plan's capacity).
size_t attn_acc_bytes(int32_t items, int32_t seqlen_max) {
  return align_up(static_cast<size_t>(items) * seqlen_max * sizeof(unsigned long long), 256);
}
size_t attn_ws_bytes(int32_t items, int32_t heads, int32_t seqlen_max) {
  if (items <= 0 || heads <= 0 || seqlen_max <= 0) return 256;
  return attn_acc_bytes(items, seqlen_max) + align_up(static_cast<size_t>(items) * sizeof(int32_t), 256);
}

// Key splits the tcgen05 kernel runs: its cluster merge takes 1, 2, 4 or 8
// (a request in between rounds down; results do not depend on the split).
int tc_splits(int requested) { return requested >= 8 ? 8 : requested >= 4 ? 4 : requested >= 2 ? 2 : 1; }

template <bool kVerify>
int launch_attn(const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mk1, const CUtensorMap& mv1,
                AttnParams& p, int grid_items, cudaStream_t stream) {
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return FDLLM_ERR_ARG;
  if (!attr[dev]) {
    if (cudaFuncSetAttribute(attn_tc_kernel<kVerify>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem) !=
            cudaSuccess ||
        cudaFuncSetAttribute(attn_tc_kernel<kVerify>, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared) != cudaSuccess)
      return FDLLM_ERR_CUDA;
    attr[dev] = true;
  }
  // one CTA = two work items; key splits as clusters of CTAs
  p.kv_splits = tc_splits(p.kv_splits);
  const dim3 grid(static_cast<unsigned>((grid_items + 1) / 2 * p.kv_splits), static_cast<unsigned>(p.n_heads), 1);
  if (launch_ex(attn_tc_kernel<kVerify>, grid, dim3(kTcThreads), kTcSmem, stream, static_cast<unsigned>(p.kv_splits),
                pdl_enabled(), mk, mv, mk1, mv1, p) != cudaSuccess)
    return FDLLM_ERR_CUDA;
  return cudaPeekAtLastError() == cudaSuccess ? FDLLM_OK : FDLLM_ERR_CUDA;
}

}  // namespace
}  // namespace fdllm

extern "C" {

int fdllm_attn_plan_capacity(int32_t n_rows, int32_t batch_size) {
  return fdllm::plan_capacity(n_rows < 0 ? 0 : n_rows, batch_size < 0 ? 0 : batch_size);
}

size_t fdllm_attn_plan_bytes(int32_t n_rows, int32_t batch_size) {
  const int cap = fdllm_attn_plan_capacity(n_rows, batch_size);
  const size_t batch = batch_size < 0 ? 0 : static_cast<size_t>(batch_size);
  return sizeof(int32_t) *
         (fdllm::kPlanHeader + static_cast<size_t>(cap) * fdllm::kPlanItem + batch * fdllm::kPlanSeq);
}

int fdllm_plan_cache_attention(const int64_t* masked_blocks, int32_t n_masked, const int64_t* tracked_blocks,
                               int32_t n_tracked, int32_t n_rows, int32_t batch_size, int32_t block_m,
                               int32_t seqlen_max, void* plan, size_t plan_bytes, cudaStream_t stream) {
  if (n_masked < 0 || n_tracked < 0 || n_rows < 0 || batch_size <= 0 || batch_size > fdllm::kPlanMaxBatch ||
      block_m <= 0 || seqlen_max <= 0 || plan == nullptr)
    return FDLLM_ERR_ARG;
  if ((n_masked > 0 && masked_blocks == nullptr) || (n_tracked > 0 && tracked_blocks == nullptr))
    return FDLLM_ERR_ARG;
  if (plan_bytes < fdllm_attn_plan_bytes(n_rows, batch_size)) return FDLLM_ERR_WORKSPACE;
  fdllm::plan_kernel<<<1, fdllm::kPlanThreads, 0, stream>>>(
      masked_blocks, n_masked, tracked_blocks, n_tracked, batch_size, block_m, seqlen_max, n_rows,
      fdllm::plan_capacity(n_rows, batch_size), static_cast<int32_t*>(plan), fdllm::status_ptr());
  return cudaPeekAtLastError() == cudaSuccess ? FDLLM_OK : FDLLM_ERR_CUDA;
}

size_t fdllm_attn_workspace_bytes(int32_t max_items, int32_t n_heads, int32_t seqlen_max) {
  return fdllm::attn_ws_bytes(max_items, n_heads, seqlen_max);
}

int fdllm_attn_cache(const void* q, void* o, const void* k_cache, const void* v_cache, const void* plan,
                     int32_t max_items, float* attn_scores, float score_scale, int32_t d_model, int32_t n_heads,
                     int32_t seqlen_max, int64_t n_slots, float softmax_scale, int32_t kv_splits,
                     const int32_t* page_table, int32_t pages_per_seq, void* workspace, size_t workspace_bytes,
                     cudaStream_t stream) {
  using namespace fdllm;
  if (n_heads <= 0 || d_model != n_heads * kHD || seqlen_max <= 0 || n_slots <= 0 || max_items < 0 ||
      kv_splits < 1 || kv_splits > 64)
    return FDLLM_ERR_ARG;
  if (page_table != nullptr &&
      (pages_per_seq <= 0 || static_cast<int64_t>(pages_per_seq) * kKeyTile < seqlen_max || n_slots < kKeyTile))
    return FDLLM_ERR_ARG;
  if (max_items == 0) return FDLLM_OK;
  const void* ptrs[] = {q, o, k_cache, v_cache, plan};
  for (const void* x : ptrs)
    if (x == nullptr || !aligned16(x)) return FDLLM_ERR_ARG;
  if (attn_scores != nullptr &&
      (workspace == nullptr || !aligned16(workspace) ||
       workspace_bytes < attn_ws_bytes(max_items, n_heads, seqlen_max)))
    return FDLLM_ERR_WORKSPACE;
  CUtensorMap mk, mv;
  int rc;
  if ((rc = make_tmap_bf16_sw128(&mk, k_cache, n_slots, d_model, d_model, kKeyTile)) != FDLLM_OK) return rc;
  if ((rc = make_tmap_bf16_sw128(&mv, v_cache, n_slots, d_model, d_model, kKeyTile)) != FDLLM_OK) return rc;
  AttnParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.o = static_cast<__nv_bfloat16*>(o);
  p.kc = static_cast<const __nv_bfloat16*>(k_cache);
  p.vc = static_cast<const __nv_bfloat16*>(v_cache);
  p.plan = static_cast<const int32_t*>(plan);
  p.scores = attn_scores;
  if (attn_scores != nullptr) {
    p.score_acc = static_cast<unsigned long long*>(workspace);
    p.score_cnt = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(workspace) + attn_acc_bytes(max_items, seqlen_max));
  }
  p.pages = page_table;
  p.pages_per_seq = page_table != nullptr ? pages_per_seq : 0;
  p.status = status_ptr();
  p.n_slots = n_slots;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.score_scale = score_scale;
  p.d_model = d_model;
  p.n_heads = n_heads;
  p.seqlen_max = seqlen_max;
  p.kv_splits = kv_splits;
  p.max_items = max_items;
  return launch_attn<false>(mk, mv, mk, mv, p, max_items, stream);
}

int fdllm_verify_attn(const void* q1, const void* k1, const void* v1, void* o, const void* k_cache,
                      const void* v_cache, const int64_t* pos_k, int64_t n_pos_k, const uint8_t* attn_mask,
                      const int32_t* verify_blocks, int32_t n_blocks, int32_t block_rows, int32_t n_rows,
                      int32_t d_model, int32_t n_heads, int64_t n_slots, float softmax_scale, int32_t kv_splits,
                      void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  using namespace fdllm;
  if (n_rows <= 0 || n_heads <= 0 || d_model != n_heads * kHD || n_blocks < 0 || block_rows <= 0 || block_rows > 1024 ||
      n_slots <= 0 || n_pos_k < 0 || kv_splits < 1 || kv_splits > 64)
    return FDLLM_ERR_ARG;
  if (n_blocks == 0) return FDLLM_OK;
  const void* ptrs[] = {q1, k1, v1, o, k_cache, v_cache, attn_mask, verify_blocks};
  for (const void* x : ptrs)
    if (x == nullptr) return FDLLM_ERR_ARG;
  if (!aligned16(q1) || !aligned16(k1) || !aligned16(v1) || !aligned16(k_cache) || !aligned16(v_cache))
    return FDLLM_ERR_ARG;
  if (n_pos_k > 0 && pos_k == nullptr) return FDLLM_ERR_ARG;
  AttnParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q1);
  p.k1 = static_cast<const __nv_bfloat16*>(k1);
  p.v1 = static_cast<const __nv_bfloat16*>(v1);
  p.o = static_cast<__nv_bfloat16*>(o);
  p.kc = static_cast<const __nv_bfloat16*>(k_cache);
  p.vc = static_cast<const __nv_bfloat16*>(v_cache);
  p.pos_k = pos_k;
  p.n_pos_k = n_pos_k;
  p.mask = attn_mask;
  p.vblocks = verify_blocks;
  p.status = status_ptr();
  p.n_slots = n_slots;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.d_model = d_model;
  p.n_heads = n_heads;
  p.kv_splits = kv_splits;
  p.n_rows = n_rows;
  p.block_rows = block_rows;
  p.row_chunks = (block_rows + kItemRows - 1) / kItemRows;
  p.n_items = n_blocks * p.row_chunks;
  // tensor maps for tiles whose keys are consecutive rows (TMA instead of a gather)
  CUtensorMap mk, mv, mk1, mv1;
  int rc;
  if ((rc = make_tmap_bf16_sw128(&mk, k_cache, n_slots, d_model, d_model, kKeyTile)) != FDLLM_OK) return rc;
  if ((rc = make_tmap_bf16_sw128(&mv, v_cache, n_slots, d_model, d_model, kKeyTile)) != FDLLM_OK) return rc;
  if ((rc = make_tmap_bf16_sw128(&mk1, k1, n_rows, d_model, d_model, kKeyTile)) != FDLLM_OK) return rc;
  if ((rc = make_tmap_bf16_sw128(&mv1, v1, n_rows, d_model, d_model, kKeyTile)) != FDLLM_OK) return rc;
  (void)workspace;  // reserved: the verify kernel needs no workspace
  (void)workspace_bytes;
  return launch_attn<true>(mk, mv, mk1, mv1, p, p.n_items, stream);
}

}  // extern "C"
