// Persistent stream-K GEMM on tcgen05 tensor cores with fused epilogues:
//
//   C[rows, cols] = A[rows, K] * B[cols, K]^T      (bf16 in, fp32 accumulate)
//
// and, instead of storing C, one of
//   kEpiQkv    RoPE on the Q and K columns with the row's slot sin/cos, Q to
//              its row, K and V to cache row pos[r] (or row-indexed), where
//              B = [W_q; W_k; W_v] is given as three tensors
//              (ref llada/flash_cache_triton.py:15-100, 255-338);
//   kEpiStore  out = bf16(C (+ residual)) (ref :618-627, 634-636: attn_out,
//              ff_out and their residual adds; the LM head);
//   kEpiSwiglu B = [W_gate; W_up] stacked (2H rows): out[:, j] =
//              bf16(bf16(silu(bf16(gate_j))) * bf16(up_j)), so the gate / up
//              activations never reach HBM (ref :628-633).
//
// Work decomposition.  A tile is 128 rows x BN columns (BN = 128 or 256
// UMMA columns).  The CTAs form one group per 128-row m-tile; each group
// covers the (column tile, k-block) space of its m-tile, one contiguous range
// per CTA (stream-K), so every SM streams the same number of k-blocks
// whatever the tile count.  CTA j of every group has the same range, so the
// groups read each weight k-block at about the same time: it comes from
// DRAM once and from L2 for the other m-tiles.  At 64 rows the kernel is
// bound by reading the weights once from HBM, at 512 rows by the tensor
// cores.  (More m-tiles than SMs: one group, m-tiles innermost.)
//
// A range starts inside a tile ("tail piece": that tile's last k-blocks),
// runs over whole tiles and ends inside a tile ("head piece": its first
// k-blocks).  Tail pieces are always a CTA's first segment: the CTA stores
// its fp32 partial accumulator to its slot of the workspace and publishes it
// with a release flag.  The CTA holding a tile's head piece (its last
// segment) is the tile's owner: it waits for the flags of the CTAs after it
// whose ranges start inside the tile (they did those k-blocks first, so the
// wait is normally already over), adds their partials in CTA order -- a fixed
// order, so results do not depend on timing -- runs the epilogue and clears
// the flags for the next call.  Every CTA of the grid is resident at once
// (grid <= SMs, one CTA per SM), and every wait is bounded.
//
// Warp roles (384 threads): warp 0 TMA producer into a ring of KSUB x 64-K
// stages (128-byte swizzle), warp 1 TMEM owner and single-thread MMA issuer
// (M = 128, N = BN) into one of two TMEM accumulators (segments alternate),
// warps 4-11 the epilogue, which overlaps the next segment's MMAs: two warps
// per TMEM lane quarter (thread = tile row), each taking every other group
// of columns, so two groups' memory traffic is in flight at once.  The
// producer / MMA warpgroup gives registers up (setmaxnreg 48) to the two
// epilogue warpgroups (224 each).
#include "common.cuh"
#include "internal.h"

namespace fdllm {

constexpr int kGBM = 128;
constexpr int kGBK = 64;
constexpr int kGThreads = 384;     // warpgroup 0: producer, MMA, 2 idle; warpgroups 1-2: epilogue
constexpr int kGEpiThreads = 256;
constexpr int kGRegsLow = 48, kGRegsHigh = 224;
static_assert(128 * kGRegsLow + 256 * kGRegsHigh <= kGThreads * 168, "setmaxnreg split");
constexpr int kGemmKernelId = 7;
constexpr int kGRingBytes = 160 * 1024;
constexpr size_t kGFlagBytes = 4096;  // one int32 flag per CTA (grid <= 1024)
constexpr int kGStageBytes = 8 * 32 * 64 * 4;  // epilogue staging: 8 warps x 32 rows x 64 fp32

enum GemmEpi { kEpiQkv = 0, kEpiStore = 1, kEpiSwiglu = 2 };

template <int BN, int XROWS, int KSUB>
struct GCfg {
  static constexpr int kASub = XROWS * kGBK * 2;  // MMA reads 128 rows; rows >= XROWS are not used
  static constexpr int kBSub = BN * kGBK * 2;
  static constexpr int kABytes = KSUB * kASub;
  static constexpr int kStageBytes = KSUB * (kASub + kBSub);
  static constexpr int kStages = kGRingBytes / kStageBytes;
  static constexpr int kBarOffset = kStages * kStageBytes;
  static constexpr int kSmem = 1024 + kBarOffset + kGStageBytes + 256;
  static constexpr int kTmemCols = 2 * BN;
  static_assert(kStages >= 2, "ring depth");
  static_assert(kSmem <= 232448, "shared memory");
};

struct GemmParams {
  int32_t groups;    // CTA groups (one per m-tile, or 1)
  int32_t n_rows;
  int32_t n_cols;    // output columns of C (QKV: 3 d; store: N; swiglu: 2 H)
  int32_t m_tiles;
  int32_t n_tiles;
  int32_t kbt;       // k-blocks (KSUB x 64) per tile
  int32_t iters;     // stream-K iterations per group: sk_tiles * kbt
  int32_t sk_tiles;  // the group's first sk_tiles tiles are split in k-blocks over its CTAs
  int32_t tiles;     // tiles per group: n_tiles (x m_tiles with one group)
  int32_t epi;
  int32_t d_model;   // QKV: columns per projection
  int32_t hidden;    // swiglu: H (first up row of the stacked weight)
  int32_t kv_by_slot;
  int64_t n_slots;
  int64_t ld_out;
  int64_t ld_res;
  __nv_bfloat16* out0;  // QKV: q; store / swiglu: out
  __nv_bfloat16* out1;  // QKV: k
  __nv_bfloat16* out2;  // QKV: v
  const __nv_bfloat16* res;
  const int64_t* pos;
  const float* sin;
  const float* cos;
  float* partials;   // [grid][BN / 4][128][4] fp32
  int32_t* flags;    // [grid]
  int32_t* status;
};

struct GSeg {
  int tile, k0, k1;
};

__device__ __forceinline__ int g_lo(int cta, int grid, int iters) {
  return static_cast<int>(static_cast<long long>(cta) * iters / grid);
}

// next segment of the range [i, hi): the k-blocks of one tile
__device__ __forceinline__ bool g_next(int& i, int hi, int kbt, GSeg& s) {
  if (i >= hi) return false;
  s.tile = i / kbt;
  s.k0 = i % kbt;
  s.k1 = s.k0 + (hi - i) < kbt ? s.k0 + (hi - i) : kbt;
  i += s.k1 - s.k0;
  return true;
}

// The work of CTA (or pair) idx of a group, in order: its even share of the
// stream-K region (the group's first sk_tiles tiles, k-block range
// [i, hi) = [g_lo(idx), g_lo(idx + 1)) of sk_tiles * kbt), then the whole tiles
// sk_tiles + idx, sk_tiles + idx + per_group, ... (data-parallel waves).
// The stream-K pieces come first so that their fix-up epilogues run while
// the whole tiles' MMAs stream; only the last whole tile's epilogue is left
// after the last MMA.
struct GIter {
  int i, hi, dp;
};

// (WAVES false: no whole-tile waves; the plan then puts every tile in the
// stream-K region, and the kernel carries none of this state)
template <bool WAVES>
__device__ __forceinline__ bool g_step(GIter& it, const GemmParams& p, int per_group, GSeg& s) {
  if (g_next(it.i, it.hi, p.kbt, s)) return true;
  if (!WAVES || it.dp >= p.tiles) return false;
  s.tile = it.dp;
  s.k0 = 0;
  s.k1 = p.kbt;
  it.dp += per_group;
  return true;
}

// whether segments follow the last one g_step returned
template <bool WAVES>
__device__ __forceinline__ bool g_more(const GIter& it, const GemmParams& p) {
  return it.i < it.hi || (WAVES && it.dp < p.tiles);
}

// Two 32-column chunks (ca, cb) with their partial sums: both TMEM loads and
// all partial loads are in flight together (one L2 latency per pair).
// Contributors [q0, q0 + n_smem) were copied (in order) into shared memory
// at `spart`; the others are read from the workspace.
template <int BN, int PR>
__device__ __forceinline__ void g_chunk2(uint32_t t_row, int ca, int cb, const GemmParams& p, int q0, int q1, int qmul,
                                         int qadd, const float4* spart, int n_smem, int r_tile, float (&va)[32],
                                         float (&vb)[32]) {
  __syncwarp();
  tmem_ld2_32x32b_x32(t_row + ca, t_row + cb, va, vb);
  for (int q = q0; q < q1; ++q) {
    const float4* part =
        q - q0 < n_smem
            ? spart + static_cast<size_t>(q - q0) * (PR * BN / 4)
            : reinterpret_cast<const float4*>(p.partials) + static_cast<size_t>(q * qmul + qadd) * (PR * BN / 4);
    float4 xa[8], xb[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      xa[j] = part[((ca >> 2) + j) * PR + r_tile];
      xb[j] = part[((cb >> 2) + j) * PR + r_tile];
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      va[4 * j] += xa[j].x;
      va[4 * j + 1] += xa[j].y;
      va[4 * j + 2] += xa[j].z;
      va[4 * j + 3] += xa[j].w;
      vb[4 * j] += xb[j].x;
      vb[4 * j + 1] += xb[j].y;
      vb[4 * j + 2] += xb[j].z;
      vb[4 * j + 3] += xb[j].w;
    }
  }
}

// Pull the rows the epilogue of a tile will read into L2 while its MMAs run
// (the epilogue's own loads are then L2 hits): the QKV row's RoPE tables
// (1 KB), or its residual row segment.
template <int BN, int EPI>
__device__ __forceinline__ void g_prefetch_epilogue(const GemmParams& p, int row, int n_tile, int64_t slot) {
  if (EPI == kEpiQkv) {
    if (slot < 0) return;
#pragma unroll
    for (int l = 0; l < 128; l += 32) {
      asm volatile("prefetch.global.L2 [%0];" ::"l"(p.sin + slot * 128 + l));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(p.cos + slot * 128 + l));
    }
  } else if (EPI == kEpiStore) {
    if (p.res == nullptr || row >= p.n_rows) return;
    const __nv_bfloat16* r = p.res + static_cast<int64_t>(row) * p.ld_res + n_tile * BN;
    const int n = min(BN, p.n_cols - n_tile * BN);
    for (int c = 0; c < n; c += 64) asm volatile("prefetch.global.L2 [%0];" ::"l"(r + c));
  }
}

// This thread's BN accumulator columns as a contributor's partial sums,
// [col / 4][row][4] fp32 over the tile's PR valid rows, so a warp's stores
// are 512 contiguous bytes.
template <int BN, int PR>
__device__ __forceinline__ void g_publish(uint32_t t_row, const GemmParams& p, int slot, int r_tile, int half,
                                          bool valid) {
  float4* part = reinterpret_cast<float4*>(p.partials) + static_cast<size_t>(slot) * (PR * BN / 4);
#pragma unroll 1
  for (int c = half * 64; c < BN; c += 128) {
    float v[32], w[32];
    __syncwarp();
    tmem_ld2_32x32b_x32(t_row + c, t_row + c + 32, v, w);  // all lanes (warp-wide)
    if (!valid) continue;
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      __stcg(part + ((c + j) >> 2) * PR + r_tile, make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]));
      __stcg(part + ((c + 32 + j) >> 2) * PR + r_tile, make_float4(w[j], w[j + 1], w[j + 2], w[j + 3]));
    }
  }
}

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ uint4 g_pack8(const float (&v)[8]) {
  uint4 u;
  u.x = pack_bf16x2(v[0], v[1]);
  u.y = pack_bf16x2(v[2], v[3]);
  u.z = pack_bf16x2(v[4], v[5]);
  u.w = pack_bf16x2(v[6], v[7]);
  return u;
}

// Per-warp staging of 32 rows x 64 fp32 columns (8 KB): the thread of row r
// writes its two 32-column chunks as 16 float4 units, unit u at position
// (u & 8) | ((u & 7) ^ (r & 7)) of the row (so the 32 rows spread over the
// banks); the warp then reads it back with several lanes per row, which makes
// the epilogue's global loads and stores row-contiguous.
__device__ __forceinline__ void g_stage_put(float4* stage, int lane, const float (&va)[32], const float (&vb)[32]) {
  float4* row = stage + lane * 16;
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    row[u ^ (lane & 7)] = make_float4(va[4 * u], va[4 * u + 1], va[4 * u + 2], va[4 * u + 3]);
    row[8 | (u ^ (lane & 7))] = make_float4(vb[4 * u], vb[4 * u + 1], vb[4 * u + 2], vb[4 * u + 3]);
  }
}
// 8 consecutive columns (units u, u + 1; u even) of staged row r
__device__ __forceinline__ void g_stage_get8(const float4* stage, int r, int u, float (&v)[8]) {
  const float4 x = stage[r * 16 + ((u & 8) | ((u & 7) ^ (r & 7)))];
  const float4 y = stage[r * 16 + (((u + 1) & 8) | (((u + 1) & 7) ^ (r & 7)))];
  v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
  v[4] = y.x; v[5] = y.y; v[6] = y.z; v[7] = y.w;
}

// Epilogue of one tile on this CTA's accumulator rows (global rows row0 +
// r), by the 8 epilogue warps: warp quarter w holds rows RQ w .. RQ w + RQ - 1
// in its TMEM lanes 0 .. RQ - 1 (RQ = 32 for M = 128 accumulators, 16 for
// M = 64, whose rows sit in the first 16 lanes of each lane quarter);
// `half` 0 / 1 takes the even / odd column groups.  `slot` is the QKV cache
// slot of this thread's row (-1: not written).  Lanes past RQ read row 0 of
// their quarter's partials and write nothing.
template <int BN, int EPI, int PR, int RQ>
__device__ __forceinline__ void g_tile_epilogue(const GemmParams& p, uint32_t t_row, float4* stage, int quarter,
                                                int half, int lane, int row0, int n_tile, int q0, int q1, int qmul,
                                                int qadd, const float4* spart, int n_smem, int64_t slot,
                                                float4* stage2) {
  const int r_tile = quarter * RQ + (lane < RQ ? lane : 0);
  const int wrow0 = row0 + quarter * RQ;  // global row of the warp's staged row 0
  if (EPI == kEpiQkv) {
    // 4 lanes per staged row: lane takes head columns c .. c + 7 (c = 32 half
    // + 8 sub) and their RoPE partners c + 64 ..; two rows per batch, their
    // table loads in flight together.  Both heads of a 256-column tile share
    // the rows' tables: with a second staging area free (`stage2`: the
    // operand ring after the CTA's last MMA) the two heads are staged
    // together and each row batch's tables are loaded once for both.
    const int sub = lane & 3;
    const int c = half * 32 + 8 * sub;
    constexpr int kHeads = BN / 128;
    const int group = (kHeads == 2 && stage2 != nullptr) ? 2 : 1;
#pragma unroll 1
    for (int h0 = 0; h0 < kHeads; h0 += group) {
#pragma unroll 1
      for (int g = 0; g < group; ++g) {
        const int hh = h0 + g;
        float va[32], vb[32];
        g_chunk2<BN, PR>(t_row, hh * 128 + half * 32, hh * 128 + 64 + half * 32, p, q0, q1, qmul, qadd, spart,
                         n_smem, r_tile, va, vb);
        g_stage_put(g == 0 ? stage : stage2, lane, va, vb);
      }
      __syncwarp();
      // the group's first head has the lowest projection: tables are needed
      // unless it is a V head
      const bool rope = (n_tile * BN + h0 * 128) / p.d_model < 2;
#pragma unroll 1
      for (int it = 0; it < RQ / 8; it += 2) {
        int64_t sl[2];
        float4 tb[2][8];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          sl[u] = __shfl_sync(0xffffffffu, slot, (it + u) * 8 + (lane >> 2));
          const int64_t sr = sl[u] < 0 ? 0 : sl[u];
          const float4* sp = reinterpret_cast<const float4*>(p.sin + sr * 128 + c);
          const float4* cp = reinterpret_cast<const float4*>(p.cos + sr * 128 + c);
          if (rope) {
            tb[u][0] = __ldg(sp);
            tb[u][1] = __ldg(sp + 1);
            tb[u][2] = __ldg(sp + 16);
            tb[u][3] = __ldg(sp + 17);
            tb[u][4] = __ldg(cp);
            tb[u][5] = __ldg(cp + 1);
            tb[u][6] = __ldg(cp + 16);
            tb[u][7] = __ldg(cp + 17);
          }
        }
#pragma unroll 1
        for (int g = 0; g < group; ++g) {
          const int n0 = n_tile * BN + (h0 + g) * 128;
          const int proj = n0 / p.d_model;
          const int hcol = n0 - proj * p.d_model;  // first column of the head in its projection
          __nv_bfloat16* out = proj == 0 ? p.out0 : (proj == 1 ? p.out1 : p.out2);
          const bool by_slot = proj > 0 && p.kv_by_slot;
          const float4* st = g == 0 ? stage : stage2;
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int rr = (it + u) * 8 + (lane >> 2);
            float x1[8], x2[8];
            g_stage_get8(st, rr, 2 * sub, x1);
            g_stage_get8(st, rr, 8 + 2 * sub, x2);
            if (sl[u] < 0) continue;
            if (proj < 2) {
              const float s1[8] = {tb[u][0].x, tb[u][0].y, tb[u][0].z, tb[u][0].w,
                                   tb[u][1].x, tb[u][1].y, tb[u][1].z, tb[u][1].w};
              const float s2[8] = {tb[u][2].x, tb[u][2].y, tb[u][2].z, tb[u][2].w,
                                   tb[u][3].x, tb[u][3].y, tb[u][3].z, tb[u][3].w};
              const float c1[8] = {tb[u][4].x, tb[u][4].y, tb[u][4].z, tb[u][4].w,
                                   tb[u][5].x, tb[u][5].y, tb[u][5].z, tb[u][5].w};
              const float c2[8] = {tb[u][6].x, tb[u][6].y, tb[u][6].z, tb[u][6].w,
                                   tb[u][7].x, tb[u][7].y, tb[u][7].z, tb[u][7].w};
#pragma unroll
              for (int k = 0; k < 8; ++k) {
                const float a1 = x1[k], a2 = x2[k];
                x1[k] = a1 * c1[k] - a2 * s1[k];
                x2[k] = a2 * c2[k] + a1 * s2[k];
              }
            }
            const int64_t orow = by_slot ? sl[u] : static_cast<int64_t>(wrow0 + rr);
            __nv_bfloat16* dst = out + orow * p.d_model + hcol + c;
            *reinterpret_cast<uint4*>(dst) = g_pack8(x1);
            *reinterpret_cast<uint4*>(dst + 64) = g_pack8(x2);
          }
        }
      }
      __syncwarp();
    }
  } else if (EPI == kEpiStore) {
#pragma unroll 1
    for (int g = half * 64; g < BN; g += 128) {
      const int col0 = n_tile * BN + g;
      if (col0 >= p.n_cols) break;  // uniform
      float va[32], vb[32];
      g_chunk2<BN, PR>(t_row, g, g + 32, p, q0, q1, qmul, qadd, spart, n_smem, r_tile, va, vb);
      g_stage_put(stage, lane, va, vb);
      __syncwarp();
      // 8 lanes per row: lane takes columns col0 + 8 sub .. + 7 of rows
      // 4 it + lane / 8; the residual loads of all 8 rows are in flight
      // together
      const int sub = lane & 7;
      const int col = col0 + 8 * sub;
      uint4 rv[8];
      if (p.res != nullptr) {
#pragma unroll
        for (int it = 0; it < RQ / 4; ++it) {
          const int row = wrow0 + it * 4 + (lane >> 3);
          rv[it] = (row < p.n_rows && col < p.n_cols)
                       ? __ldg(reinterpret_cast<const uint4*>(p.res + static_cast<int64_t>(row) * p.ld_res + col))
                       : make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int it = 0; it < RQ / 4; ++it) {
        const int rr = it * 4 + (lane >> 3);
        const int row = wrow0 + rr;
        float v[8];
        g_stage_get8(stage, rr, 2 * sub, v);
        if (row >= p.n_rows || col >= p.n_cols) continue;
        if (p.res != nullptr) {
          const uint32_t w[4] = {rv[it].x, rv[it].y, rv[it].z, rv[it].w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[k]));
            v[2 * k] += f.x;
            v[2 * k + 1] += f.y;
          }
        }
        *reinterpret_cast<uint4*>(p.out0 + static_cast<int64_t>(row) * p.ld_out + col) = g_pack8(v);
      }
      __syncwarp();
    }
  } else {
    // SwiGLU: accumulator columns [0, BN/2) are gate, [BN/2, BN) the matching up
#pragma unroll 1
    for (int c0 = half * 32; c0 < BN / 2; c0 += 64) {
      float gv[32], uv[32];
      g_chunk2<BN, PR>(t_row, c0, BN / 2 + c0, p, q0, q1, qmul, qadd, spart, n_smem, r_tile, gv, uv);
      g_stage_put(stage, lane, gv, uv);
      __syncwarp();
      const int sub = lane & 3;
      const int col = n_tile * (BN / 2) + c0 + 8 * sub;
#pragma unroll 1
      for (int it = 0; it < RQ / 8; ++it) {
        const int rr = it * 8 + (lane >> 2);
        const int row = wrow0 + rr;
        float g8[8], u8[8];
        g_stage_get8(stage, rr, 2 * sub, g8);
        g_stage_get8(stage, rr, 8 + 2 * sub, u8);
        if (row >= p.n_rows) continue;
        // silu with the fast exp / divide intrinsics: their few-ulp fp32 error
        // sits far below the bf16 rounding that follows, and the IEEE forms
        // serialise into ~140 cycles per element here
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float gb = bf16_round(g8[k]);
          g8[k] = bf16_round(__fdividef(gb, 1.f + __expf(-gb))) * bf16_round(u8[k]);
        }
        *reinterpret_cast<uint4*>(p.out0 + static_cast<int64_t>(row) * p.ld_out + col) = g_pack8(g8);
      }
      __syncwarp();
    }
  }
}

// Owner fix-up: copy the partial sums of contributors [q0, q0 + n) into the
// operand ring at `ring` (idle then: a head piece is its CTA's last segment,
// and every MMA that read the ring has completed) with bulk copies on
// `bar`, by one thread; the epilogue then reads them from shared memory.
template <int BN, int PR>
__device__ __forceinline__ void g_fetch_partials(const GemmParams& p, uint8_t* ring, int q0, int n, int qmul, int qadd,
                                                 uint64_t* bar) {
  constexpr uint32_t kSlot = PR * BN * 4;
  constexpr uint32_t kPiece = kSlot < 32 * 1024 ? kSlot : 32 * 1024;
  mbar_arrive_expect_tx(bar, static_cast<uint32_t>(n) * kSlot);
  for (int j = 0; j < n; ++j) {
    const uint8_t* src = reinterpret_cast<const uint8_t*>(p.partials) + static_cast<size_t>((q0 + j) * qmul + qadd) * kSlot;
    for (uint32_t off = 0; off < kSlot; off += kPiece) bulk_load(ring + j * kSlot + off, src + off, kPiece, bar);
  }
}

// Cache slot of this thread's row for the QKV epilogue (-1: no row / bad slot).
__device__ __forceinline__ int64_t g_qkv_slot(const GemmParams& p, int row) {
  if (row >= p.n_rows) return -1;
  const int64_t s = p.pos[row];
  if (s < 0 || s >= p.n_slots) {
    report(p.status, FDLLM_ERR_INDEX, row, kGemmKernelId);
    return -1;
  }
  return s;
}

// B rows of column tile n_tile for the load of CTA `rank` of a pair (rank 0
// for a single CTA; `rows` = B rows per CTA): QKV picks the projection's map.
template <int EPI>
__device__ __forceinline__ const CUtensorMap* g_b_coord(const GemmParams& p, int n_tile, int tile_cols, int rank,
                                                       int rows, const CUtensorMap* m0, const CUtensorMap* m1,
                                                       const CUtensorMap* m2, int& b_row) {
  if (EPI == kEpiQkv) {
    const int n0 = n_tile * tile_cols;
    const int proj = n0 / p.d_model;
    b_row = n0 - proj * p.d_model + rank * rows;
    return proj == 0 ? m0 : (proj == 1 ? m1 : m2);
  }
  if (EPI == kEpiSwiglu) {
    b_row = n_tile * (tile_cols / 2) + (rank ? p.hidden : 0);
    return m0;
  }
  b_row = n_tile * tile_cols + rank * rows;
  return m0;
}

template <int BN, int XROWS, int KSUB, int EPI>
__global__ void __launch_bounds__(kGThreads, 1)
    gemm_sk_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b0,
                   const __grid_constant__ CUtensorMap map_b1, const __grid_constant__ CUtensorMap map_b2,
                   const GemmParams p) {
  using C = GCfg<BN, XROWS, KSUB>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float4* stage_all = reinterpret_cast<float4*>(smem + C::kBarOffset);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOffset + kGStageBytes);
  uint64_t* empty = full + C::kStages;
  uint64_t* acc_full = empty + C::kStages;  // [2] MMA -> epilogue
  uint64_t* acc_empty = acc_full + 2;       // [2] epilogue (4 warps) -> MMA
  uint64_t* fix_bar = acc_empty + 2;        // owner fix-up: contributors' partials in the ring
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(fix_bar + 1);
  volatile int32_t* abort_flag = reinterpret_cast<volatile int32_t*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const int per_group = gridDim.x / p.groups;
  const int group = cta / per_group;  // the m-tile (one group: m-tiles innermost in the tile index)
  const int idx = cta % per_group;    // rank within the group
  const int lo = g_lo(idx, per_group, p.iters);  // stream-K range
  const int hi = g_lo(idx + 1, per_group, p.iters);
  const int m_tiles_in = p.groups > 1 ? 1 : p.m_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 8);  // 8 epilogue warps
    }
    mbar_init(fix_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b0);
    if (EPI == kEpiQkv) {
      tma_prefetch_desc(&map_b1);
      tma_prefetch_desc(&map_b2);
    }
  }
  if (warp == 1) tmem_alloc(tmem_slot, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  constexpr uint32_t kTx = static_cast<uint32_t>(C::kStageBytes);
  // B (weights: never written by the kernel before) of the stages that need
  // no free slot, requested before the programmatic-launch wait so its
  // latency overlaps the tail of the kernel before; A comes from that kernel
  auto load_b = [&](int n_tile, int kb, int s) {
    int b_row = 0;
    const CUtensorMap* map_b = g_b_coord<EPI>(p, n_tile, BN, 0, BN, &map_b0, &map_b1, &map_b2, b_row);
    uint8_t* b0 = smem + s * C::kStageBytes + C::kABytes;
#pragma unroll
    for (int sub = 0; sub < KSUB; ++sub) {
      const int kx = (kb * KSUB + sub) * kGBK;
      uint8_t* b = b0 + sub * C::kBSub;
      tma_load_2d(b, map_b, kx, b_row, &full[s]);
      if (EPI == kEpiSwiglu) tma_load_2d(b + (BN / 2) * 128, map_b, kx, p.hidden + b_row, &full[s]);
    }
  };
  uint32_t n_pre = 0;
  if (warp == 0 && lane == 0) {
    GIter it{lo, hi, p.sk_tiles + idx};
    GSeg sg;
    while (n_pre < static_cast<uint32_t>(C::kStages) && g_step<false>(it, p, per_group, sg))
      for (int kb = sg.k0; kb < sg.k1 && n_pre < static_cast<uint32_t>(C::kStages); ++kb, ++n_pre) {
        mbar_arrive_expect_tx(&full[n_pre], kTx);
        load_b(sg.tile / m_tiles_in, kb, static_cast<int>(n_pre));
      }
  }
  pdl_wait();
  pdl_launch_dependents();

  if (warp < 4) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kGRegsLow));
  if (warp == 0) {
    // ------------------------------------------------------ TMA producer --
    if (lane == 0) {
      uint32_t g = 0;
      bool ok = true;
      GIter it{lo, hi, p.sk_tiles + idx};
      GSeg sg;
      while (ok && g_step<false>(it, p, per_group, sg)) {
        const int m_tile = p.groups > 1 ? group : sg.tile % m_tiles_in, n_tile = sg.tile / m_tiles_in;
        for (int kb = sg.k0; kb < sg.k1; ++kb, ++g) {
          const int s = g % C::kStages;
          const uint32_t ph = (g / C::kStages) & 1;
          const bool pre = g < n_pre;  // B already requested, tx already expected
          if (g >= static_cast<uint32_t>(C::kStages) && !mbar_wait(&empty[s], ph ^ 1, p.status, kGemmKernelId)) {
            ok = false;
            break;
          }
          uint8_t* a0 = smem + s * C::kStageBytes;
          if (!pre) mbar_arrive_expect_tx(&full[s], kTx);
#pragma unroll
          for (int sub = 0; sub < KSUB; ++sub)
            tma_load_2d(a0 + sub * C::kASub, &map_a, (kb * KSUB + sub) * kGBK, m_tile * kGBM, &full[s]);
          if (!pre) load_b(n_tile, kb, s);
        }
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------- MMA issuer --
    if (lane == 0) {
      // M = 64 UMMAs for 64-row A tiles (no idle accumulator rows)
      constexpr uint32_t idesc = umma_idesc_bf16(XROWS == 64 ? 64 : kGBM, BN);
      uint32_t g = 0;
      int seg = 0;
      bool ok = true;
      GIter it{lo, hi, p.sk_tiles + idx};
      GSeg sg;
      while (ok && g_step<false>(it, p, per_group, sg)) {
        const int acc = seg & 1;
        if (seg >= 2 && !mbar_wait(&acc_empty[acc], ((seg >> 1) & 1) ^ 1, p.status, kGemmKernelId)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = sg.k0; kb < sg.k1; ++kb, ++g) {
          const int s = g % C::kStages;
          const uint32_t ph = (g / C::kStages) & 1;
          if (!mbar_wait(&full[s], ph, p.status, kGemmKernelId)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* a0 = smem + s * C::kStageBytes;
#pragma unroll
          for (int sub = 0; sub < KSUB; ++sub) {
            const uint64_t da = umma_desc_kmajor_sw128(smem_u32(a0 + sub * C::kASub));
            const uint64_t db = umma_desc_kmajor_sw128(smem_u32(a0 + C::kABytes + sub * C::kBSub));
#pragma unroll
            for (int k = 0; k < kGBK / 16; ++k)
              umma_bf16(d_tmem, da + 2 * k, db + 2 * k, idesc, (kb > sg.k0 || sub > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&acc_full[acc]);
        ++seg;
      }
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kGRegsHigh));
    // ---------------------------------------------------------- epilogue --
    // accumulator rows per TMEM lane quarter: 32 (M = 128) or 16 (M = 64,
    // lanes 0-15 of each quarter)
    constexpr int kRQ = XROWS == 64 ? 16 : 32;
    const int quarter = warp & 3;
    const int half = (warp - 4) >> 2;
    const bool row_lane = lane < kRQ;
    const int r_tile = quarter * kRQ + (row_lane ? lane : 0);
    const int ep_tid = threadIdx.x - 128;
    float4* stage = stage_all + (warp - 4) * (32 * 16);
    int seg = 0;
    GIter it{lo, hi, p.sk_tiles + idx};
    GSeg sg;
    while (g_step<false>(it, p, per_group, sg)) {
      const int acc = seg & 1;
      const int m_tile = p.groups > 1 ? group : sg.tile % m_tiles_in, n_tile = sg.tile / m_tiles_in;
      const int row0 = m_tile * kGBM;
      const uint32_t t_row = tmem_base + acc * BN + (static_cast<uint32_t>(quarter * 32) << 16);
      // the QKV epilogue's slot, fetched while the MMAs run
      const int64_t slot = (EPI == kEpiQkv && sg.k0 == 0 && row_lane) ? g_qkv_slot(p, row0 + r_tile) : -1;
      if (sg.k0 == 0 && half == 0 && row_lane) g_prefetch_epilogue<BN, EPI>(p, row0 + r_tile, n_tile, slot);
      // every epilogue thread reaches the named barriers (all waits are
      // bounded), so the decisions below are uniform over the 4 warps
      if (!mbar_wait(&acc_full[acc], (seg >> 1) & 1, p.status, kGemmKernelId)) *abort_flag = 1;
      asm volatile("bar.sync 1, 256;" ::: "memory");
      if (*abort_flag != 0) break;
      tc_fence_after();
      if (sg.k0 > 0) {
        // tail piece (this CTA's first segment): publish the partial sums of
        // the tile's XROWS valid rows; after the barrier one thread's release
        // store (cumulative over the CTA's stores ordered by the barrier)
        // raises the flag
        g_publish<BN, XROWS>(t_row, p, cta, r_tile, half, row_lane);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[acc]);
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (ep_tid == 0) st_release_gpu(p.flags + cta, 1);
        ++seg;
        continue;
      }
      // whole tile, or the owner's head piece: wait for the contributors
      int q_end = cta + 1;  // contributors: the next CTAs of the group
      if (sg.k1 < p.kbt) {
        const int t_end = (sg.tile + 1) * p.kbt;
        while (q_end - group * per_group < per_group && g_lo(q_end - group * per_group, per_group, p.iters) < t_end)
          ++q_end;
        bool ok = true;
        if (ep_tid == 0)
          for (int q = cta + 1; q < q_end && ok; ++q) ok = flag_wait_set(p.flags + q, p.status, kGemmKernelId);
        if (!ok) *abort_flag = 1;
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (*abort_flag != 0) break;
      }
      // contributors' partials go to the operand ring when it is idle (this
      // is the CTA's last segment); otherwise they are read from the workspace
      int n_smem = 0;
      if (q_end > cta + 1 && !g_more<false>(it, p)) {
        n_smem = min(q_end - cta - 1, C::kBarOffset / (XROWS * BN * 4));
        if (ep_tid == 0) g_fetch_partials<BN, XROWS>(p, smem, cta + 1, n_smem, 1, 0, fix_bar);
        if (!mbar_wait(fix_bar, 0, p.status, kGemmKernelId)) n_smem = 0;  // (recorded; sums then incomplete)
      }
      // after the CTA's last MMA the operand ring is free unless it holds
      // contributors' partials: a second staging area for the QKV epilogue
      float4* stage2 = (!g_more<false>(it, p) && q_end == cta + 1)
                           ? reinterpret_cast<float4*>(smem) + (warp - 4) * (32 * 16) : nullptr;
      g_tile_epilogue<BN, EPI, XROWS, kRQ>(p, t_row, stage, quarter, half, lane, row0, n_tile, cta + 1, q_end, 1, 0,
                                           reinterpret_cast<const float4*>(smem), n_smem, slot, stage2);
      // every column of this accumulator has been read
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
      if (q_end > cta + 1) {
        // every epilogue thread has read the partials: clear their flags
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (ep_tid == 0)
          for (int q = cta + 1; q < q_end; ++q) p.flags[q] = 0;
      }
      ++seg;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// CTA-pair variant (more than 128 rows): clusters of two CTAs compute
// 256-row x 256-column tiles with 2-SM UMMAs (cta_group::2, M = 256): CTA r
// loads rows 128 r .. 128 r + 127 of the tile's A rows and B rows
// 128 r .. 128 r + 127 of its 256 columns, and holds its 128 output rows x 256
// columns in its own TMEM.  Each SM then moves 32 KB of operands per 64-K
// step for 4.2 MFLOP (a single-CTA 128 x 256 tile: 48 KB), within what one
// SM pulls from L2.  Stream-K as above, over pairs: pair j of every m-tile
// group has the same range; a contributor pair's CTAs publish their partial
// sums and flags separately, and each CTA of the owner pair adds those of
// its rank.  The leader's `full` barrier expects both CTAs' bytes; stage,
// accumulator and TMEM-free completions go to both CTAs.
// ---------------------------------------------------------------------------
template <int KSUB>
struct G2Cfg {
  static constexpr int kSub = kGBM * kGBK * 2;      // 128 rows x 64 K (A, or this CTA's half of B)
  static constexpr int kABytes = KSUB * kSub;
  static constexpr int kStageBytes = 2 * KSUB * kSub;
  static constexpr int kStages = kGRingBytes / kStageBytes;
  static constexpr int kBarOffset = kStages * kStageBytes;
  static constexpr int kSmem = 1024 + kBarOffset + kGStageBytes + 256;
  static_assert(kSmem <= 232448, "shared memory");
};

template <int KSUB, int EPI, bool WAVES>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGThreads, 1)
    gemm_sk2_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b0,
                    const __grid_constant__ CUtensorMap map_b1, const __grid_constant__ CUtensorMap map_b2,
                    const GemmParams p) {
  using C = G2Cfg<KSUB>;
  constexpr int BN = 256;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float4* stage_all = reinterpret_cast<float4*>(smem + C::kBarOffset);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOffset + kGStageBytes);
  uint64_t* empty = full + C::kStages;
  uint64_t* acc_full = empty + C::kStages;  // [2] leader's MMA -> both CTAs' epilogues
  uint64_t* acc_empty = acc_full + 2;       // [2] both epilogues (8 warps) -> leader's MMA
  uint64_t* fix_bar = acc_empty + 2;        // owner fix-up: contributors' partials in the ring
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(fix_bar + 1);
  volatile int32_t* abort_flag = reinterpret_cast<volatile int32_t*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const uint32_t rank = cluster_ctarank();
  const int pair = cta >> 1;
  const int n_pairs = gridDim.x >> 1;
  const int per_group = n_pairs / p.groups;
  const int group = pair / per_group;
  const int idx = pair % per_group;
  const int lo = g_lo(idx, per_group, p.iters);
  const int hi = g_lo(idx + 1, per_group, p.iters);
  const int m_tiles_in = p.groups > 1 ? 1 : p.m_tiles;  // m-tiles of 256 rows

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);   // the leader's expect_tx arrival (used on the leader)
      mbar_init(&empty[s], 1);  // the leader's commit
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 16);  // 8 epilogue warps x 2 CTAs (used on the leader)
    }
    mbar_init(fix_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b0);
    if (EPI == kEpiQkv) {
      tma_prefetch_desc(&map_b1);
      tma_prefetch_desc(&map_b2);
    }
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, 2 * BN);
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before any remote arrival
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // B (weights) of the stages that need no free slot, requested before the
  // programmatic-launch wait (see the single-CTA kernel); A after it
  auto load_b = [&](int n_tile, int kb, int s) {
    int b_row = 0;
    const CUtensorMap* map_b =
        g_b_coord<EPI>(p, n_tile, BN, static_cast<int>(rank), kGBM, &map_b0, &map_b1, &map_b2, b_row);
    const uint32_t bar = mapa_shared(&full[s], 0);
#pragma unroll
    for (int sub = 0; sub < KSUB; ++sub)
      tma_load_2d_pair(smem + s * C::kStageBytes + C::kABytes + sub * C::kSub, map_b, (kb * KSUB + sub) * kGBK, b_row,
                       bar);
  };
  uint32_t n_pre = 0;
  if (warp == 0 && lane == 0) {
    GIter it{lo, hi, p.sk_tiles + idx};
    GSeg sg;
    while (n_pre < static_cast<uint32_t>(C::kStages) && g_step<WAVES>(it, p, per_group, sg))
      for (int kb = sg.k0; kb < sg.k1 && n_pre < static_cast<uint32_t>(C::kStages); ++kb, ++n_pre) {
        if (rank == 0) mbar_arrive_expect_tx(&full[n_pre], 2u * C::kStageBytes);
        load_b(sg.tile / m_tiles_in, kb, static_cast<int>(n_pre));
      }
  }
  pdl_wait();
  pdl_launch_dependents();

  if (warp < 4) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kGRegsLow));
  if (warp == 0) {
    // ------------------------------------------------------ TMA producer --
    if (lane == 0) {
      uint32_t g = 0;
      bool ok = true;
      GIter it{lo, hi, p.sk_tiles + idx};
      GSeg sg;
      while (ok && g_step<WAVES>(it, p, per_group, sg)) {
        const int m_tile = p.groups > 1 ? group : sg.tile % m_tiles_in, n_tile = sg.tile / m_tiles_in;
        const int a_row = m_tile * 2 * kGBM + static_cast<int>(rank) * kGBM;
        for (int kb = sg.k0; kb < sg.k1; ++kb, ++g) {
          const int s = g % C::kStages;
          const uint32_t ph = (g / C::kStages) & 1;
          const bool pre = g < n_pre;  // B already requested, tx already expected
          if (g >= static_cast<uint32_t>(C::kStages) && !mbar_wait(&empty[s], ph ^ 1, p.status, kGemmKernelId)) {
            ok = false;
            break;
          }
          uint8_t* a0 = smem + s * C::kStageBytes;
          const uint32_t bar = mapa_shared(&full[s], 0);
          if (rank == 0 && !pre) mbar_arrive_expect_tx(&full[s], 2u * C::kStageBytes);
#pragma unroll
          for (int sub = 0; sub < KSUB; ++sub)
            tma_load_2d_pair(a0 + sub * C::kSub, &map_a, (kb * KSUB + sub) * kGBK, a_row, bar);
          if (!pre) load_b(n_tile, kb, s);
        }
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------- MMA issuer (leader only) --
    if (rank == 0 && lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(2 * kGBM, BN);
      uint32_t g = 0;
      int seg = 0;
      bool ok = true;
      GIter it{lo, hi, p.sk_tiles + idx};
      GSeg sg;
      while (ok && g_step<WAVES>(it, p, per_group, sg)) {
        const int acc = seg & 1;
        if (seg >= 2 && !mbar_wait(&acc_empty[acc], ((seg >> 1) & 1) ^ 1, p.status, kGemmKernelId)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = sg.k0; kb < sg.k1; ++kb, ++g) {
          const int s = g % C::kStages;
          const uint32_t ph = (g / C::kStages) & 1;
          if (!mbar_wait(&full[s], ph, p.status, kGemmKernelId)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* a0 = smem + s * C::kStageBytes;
#pragma unroll
          for (int sub = 0; sub < KSUB; ++sub) {
            const uint64_t da = umma_desc_kmajor_sw128(smem_u32(a0 + sub * C::kSub));
            const uint64_t db = umma_desc_kmajor_sw128(smem_u32(a0 + C::kABytes + sub * C::kSub));
#pragma unroll
            for (int k = 0; k < kGBK / 16; ++k)
              umma_bf16_pair(d_tmem, da + 2 * k, db + 2 * k, idesc, (kb > sg.k0 || sub > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit_pair(mapa_shared(&empty[s], 0));
          umma_commit_pair(mapa_shared(&empty[s], 1));
        }
        if (!ok) break;
        umma_commit_pair(mapa_shared(&acc_full[acc], 0));
        umma_commit_pair(mapa_shared(&acc_full[acc], 1));
        ++seg;
      }
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kGRegsHigh));
    // ---------------------------------------------------------- epilogue --
    const int quarter = warp & 3;
    const int half = (warp - 4) >> 2;
    const int r_tile = quarter * 32 + lane;
    const int ep_tid = threadIdx.x - 128;
    float4* stage = stage_all + (warp - 4) * (32 * 16);
    const uint32_t acc_empty_leader[2] = {mapa_shared(&acc_empty[0], 0), mapa_shared(&acc_empty[1], 0)};
    int seg = 0;
    GIter it{lo, hi, p.sk_tiles + idx};
    GSeg sg;
    while (g_step<WAVES>(it, p, per_group, sg)) {
      const int acc = seg & 1;
      const int m_tile = p.groups > 1 ? group : sg.tile % m_tiles_in, n_tile = sg.tile / m_tiles_in;
      const int row0 = m_tile * 2 * kGBM + static_cast<int>(rank) * kGBM;
      const uint32_t t_row = tmem_base + acc * BN + (static_cast<uint32_t>(quarter * 32) << 16);
      const int64_t slot = (EPI == kEpiQkv && sg.k0 == 0) ? g_qkv_slot(p, row0 + r_tile) : -1;
      if (sg.k0 == 0 && half == 0) g_prefetch_epilogue<BN, EPI>(p, row0 + r_tile, n_tile, slot);
      if (!mbar_wait(&acc_full[acc], (seg >> 1) & 1, p.status, kGemmKernelId)) *abort_flag = 1;
      asm volatile("bar.sync 1, 256;" ::: "memory");
      if (*abort_flag != 0) break;
      tc_fence_after();
      if (sg.k0 > 0) {
        g_publish<BN, kGBM>(t_row, p, cta, r_tile, half, true);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(acc_empty_leader[acc]);
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (ep_tid == 0) st_release_gpu(p.flags + cta, 1);
        ++seg;
        continue;
      }
      int q_end = pair + 1;  // contributor pairs: the next pairs of the group
      if (sg.k1 < p.kbt) {
        const int t_end = (sg.tile + 1) * p.kbt;
        while (q_end - group * per_group < per_group && g_lo(q_end - group * per_group, per_group, p.iters) < t_end)
          ++q_end;
        bool ok = true;
        if (ep_tid == 0)
          for (int q = pair + 1; q < q_end && ok; ++q)
            ok = flag_wait_set(p.flags + 2 * q + static_cast<int>(rank), p.status, kGemmKernelId);
        if (!ok) *abort_flag = 1;
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (*abort_flag != 0) break;
      }
      int n_smem = 0;
      if (q_end > pair + 1 && !g_more<WAVES>(it, p)) {
        n_smem = min(q_end - pair - 1, C::kBarOffset / (kGBM * BN * 4));
        if (ep_tid == 0) g_fetch_partials<BN, kGBM>(p, smem, pair + 1, n_smem, 2, static_cast<int>(rank), fix_bar);
        if (!mbar_wait(fix_bar, 0, p.status, kGemmKernelId)) n_smem = 0;  // (recorded; sums then incomplete)
      }
      // after the pair's last MMA (its completion reached both CTAs) the
      // operand ring is free unless it holds contributors' partials
      float4* stage2 = (!g_more<WAVES>(it, p) && q_end == pair + 1)
                           ? reinterpret_cast<float4*>(smem) + (warp - 4) * (32 * 16) : nullptr;
      g_tile_epilogue<BN, EPI, kGBM, 32>(p, t_row, stage, quarter, half, lane, row0, n_tile, pair + 1, q_end, 2,
                               static_cast<int>(rank), reinterpret_cast<const float4*>(smem), n_smem, slot, stage2);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty_leader[acc]);
      if (q_end > pair + 1) {
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (ep_tid == 0)
          for (int q = pair + 1; q < q_end; ++q) p.flags[2 * q + static_cast<int>(rank)] = 0;
      }
      ++seg;
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the leader's MMAs read both CTAs' shared memory until here
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 2 * BN);
  }
}

namespace {

struct GemmPlan {
  bool pair;  // CTA-pair kernel (256-row tiles)
  int bn, xrows, ksub, grid, groups;
  int m_tiles, n_tiles, kbt, iters, sk_tiles, tiles;
};

// Plan overrides for tuning and tests (fdllm_gemm_set_plan): 0 / -1 = automatic.
struct GemmOverride {
  int bn, ksub, grid, pair, dp;
};
GemmOverride& gemm_override() {
  static GemmOverride o{env_int("FDLLM_GEMM_BN", 0), env_int("FDLLM_GEMM_KSUB", 0), env_int("FDLLM_GEMM_GRID", 0),
                        env_int("FDLLM_GEMM_PAIR", -1), env_int("FDLLM_GEMM_DP", 0)};
  return o;
}

// Resident 2-CTA clusters of a pair-kernel configuration (an SM count that
// is odd within a GPC leaves SMs out); cached per device and configuration.
template <int KSUB, int EPI>
int g2_max_pairs() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (cache[dev] == 0) {
    using C = G2Cfg<KSUB>;
    if (cudaFuncSetAttribute(gemm_sk2_kernel<KSUB, EPI, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::kSmem) != cudaSuccess ||
        cudaFuncSetAttribute(gemm_sk2_kernel<KSUB, EPI, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::kSmem) != cudaSuccess)
      return 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(kGThreads, 1, 1);
    cfg.dynamicSmemBytes = C::kSmem;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_sk2_kernel<KSUB, EPI, false>, &cfg) != cudaSuccess || n <= 0)
      return 0;
    cache[dev] = n;
  }
  return cache[dev];
}

int g2_max_pairs_for(int epi, int ksub) {
  if (epi == kEpiQkv) return ksub == 2 ? g2_max_pairs<2, kEpiQkv>() : g2_max_pairs<1, kEpiQkv>();
  if (epi == kEpiStore) return ksub == 2 ? g2_max_pairs<2, kEpiStore>() : g2_max_pairs<1, kEpiStore>();
  return ksub == 2 ? g2_max_pairs<2, kEpiSwiglu>() : g2_max_pairs<1, kEpiSwiglu>();
}

// Up to 128 rows: single CTAs with 128-column tiles, stream-K (the kernel
// streams weights from HBM; narrower tiles give more tiles, so fewer
// stream-K pieces per tile).  Above: CTA pairs with 256 x 256 tiles, stream-K
// (bound by operand ingress per SM, which a pair halves for B) -- except
// short-K problems whose 128 x 128 tiles fit the grid at once: single CTAs,
// one whole tile each with no fix-ups when the tiles nearly fill the grid
// (attn_out: 4096 x 4096 at 4 x 128 rows), stream-K otherwise.  Ring stages: two 64-K boxes (256 B of every operand row per
// request) for 64-row single CTAs, one 64-K box elsewhere.
GemmPlan plan_gemm(int epi, int32_t n_rows, int32_t n_cols, int32_t k_dim, int32_t d_model) {
  GemmPlan pl{};
  const GemmOverride& ov = gemm_override();
  const int out_cols = epi == kEpiSwiglu ? n_cols / 2 : n_cols;
  bool dp = ov.dp == 1;
  if (ov.pair < 0 && ov.dp == 0 && n_rows > kGBM && k_dim <= 4096) {
    // whole tiles only when they nearly fill one wave: with fewer, stream-K
    // over all SMs measured faster (attn_out 4096 x 4096: 64 tiles at 256
    // rows 20.1 vs 23.7 us, 96 at 384 rows 22.7 vs 24.6; 128 at 448-512
    // rows 24.6 vs 26.2 with whole tiles)
    const long long tiles128 = static_cast<long long>((n_rows + kGBM - 1) / kGBM) *
                               ((out_cols + (epi == kEpiSwiglu ? 63 : 127)) / (epi == kEpiSwiglu ? 64 : 128));
    if (tiles128 <= sm_count() && 5 * tiles128 >= 4ll * sm_count()) dp = true;
  }
  pl.pair = ov.pair < 0 ? (n_rows > kGBM && !dp) : ov.pair != 0;
  if (epi == kEpiQkv && d_model % 256 != 0) pl.pair = false;  // a pair tile holds two heads of one projection
  int bn;
  if (pl.pair) {
    bn = 256;
    pl.xrows = kGBM;
    pl.m_tiles = (n_rows + 2 * kGBM - 1) / (2 * kGBM);
  } else {
    bn = ov.bn == 128 || ov.bn == 256 ? ov.bn : 128;
    if (epi == kEpiQkv && d_model % bn != 0) bn = 128;
    pl.xrows = n_rows <= 64 ? 64 : kGBM;
    pl.m_tiles = (n_rows + kGBM - 1) / kGBM;
  }
  int ksub = ov.ksub == 1 || ov.ksub == 2 ? ov.ksub : (!pl.pair && pl.xrows == 64 ? 2 : 1);
  if (!pl.pair && bn == 256 && pl.xrows == kGBM) ksub = 1;  // a 96 KB stage leaves one stage
  if (k_dim % (kGBK * ksub) != 0) ksub = 1;
  pl.ksub = ksub;
  pl.kbt = k_dim / (kGBK * ksub);
  pl.bn = bn;
  const int out_per_tile = epi == kEpiSwiglu ? bn / 2 : bn;
  pl.n_tiles = (out_cols + out_per_tile - 1) / out_per_tile;
  // every CTA must be resident at once (owners wait for contributors): at
  // most one CTA per SM, or the resident pairs
  int units = pl.pair ? g2_max_pairs_for(epi, ksub) : sm_count();
  if (units <= 0) units = pl.pair ? sm_count() / 2 : sm_count();
  if (ov.grid > 0 && ov.grid < units) units = ov.grid;
  if (units > (pl.pair ? 512 : 1024)) units = pl.pair ? 512 : 1024;
  pl.groups = pl.m_tiles <= units ? pl.m_tiles : 1;
  const long long iters = static_cast<long long>(pl.groups > 1 ? 1 : pl.m_tiles) * pl.n_tiles * pl.kbt;
  if (iters > (1ll << 30)) {
    pl.iters = -1;
    return pl;
  }
  int per_group = units / pl.groups;
  if (per_group > iters) per_group = static_cast<int>(iters);
  // data-parallel: at most one whole tile per CTA (no fix-ups) when the
  // tiles fit the grid
  const int tiles_per_group = pl.groups > 1 ? pl.n_tiles : pl.m_tiles * pl.n_tiles;
  if (dp && tiles_per_group <= per_group) per_group = tiles_per_group;
  // CTA pairs: whole-tile waves plus a stream-K region of the remaining
  // tiles (split first, so only the last whole tile's epilogue follows the
  // last MMA; measured 4 and 3 us faster for the QKV and MLP GEMMs at 512
  // rows; single CTAs, whose tile epilogues are shorter, measured no gain);
  // a region of fewer than per_group / 8 tiles (pieces under 1/8 of a tile)
  // takes one wave of whole tiles in with it (so does one with fewer
  // k-blocks than CTAs: every CTA's range must be non-empty).  dp = 2: all
  // tiles stream-K.
  int sk_tiles = tiles_per_group;
  if (pl.pair && ov.dp != 2 && tiles_per_group >= per_group) {
    sk_tiles = tiles_per_group % per_group;
    if (sk_tiles > 0 && (8 * sk_tiles < per_group || static_cast<long long>(sk_tiles) * pl.kbt < per_group))
      sk_tiles += per_group;
  }
  pl.sk_tiles = sk_tiles;
  pl.tiles = tiles_per_group;
  pl.iters = sk_tiles * pl.kbt;
  pl.grid = per_group * pl.groups * (pl.pair ? 2 : 1);
  return pl;
}

size_t gemm_ws_bytes(const GemmPlan& pl) {
  return kGFlagBytes + static_cast<size_t>(pl.grid) * kGBM * pl.bn * sizeof(float);
}

template <int BN, int XROWS, int KSUB, int EPI>
int launch_gemm_cfg(const CUtensorMap& ma, const CUtensorMap& mb0, const CUtensorMap& mb1, const CUtensorMap& mb2,
                    const GemmParams& p, int grid, cudaStream_t stream) {
  using C = GCfg<BN, XROWS, KSUB>;
  static bool attr_set[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return FDLLM_ERR_CUDA;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(gemm_sk_kernel<BN, XROWS, KSUB, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::kSmem) != cudaSuccess)
      return FDLLM_ERR_CUDA;
    attr_set[dev] = true;
  }
  if (launch_ex(gemm_sk_kernel<BN, XROWS, KSUB, EPI>, dim3(grid), dim3(kGThreads), C::kSmem, stream, 1,
                pdl_enabled(), ma, mb0, mb1, mb2, p) != cudaSuccess)
    return FDLLM_ERR_CUDA;
  return cudaPeekAtLastError() == cudaSuccess ? FDLLM_OK : FDLLM_ERR_CUDA;
}

template <int KSUB, int EPI>
int launch_gemm2_cfg(const CUtensorMap& ma, const CUtensorMap& mb0, const CUtensorMap& mb1, const CUtensorMap& mb2,
                     const GemmParams& p, int grid, cudaStream_t stream) {
  using C = G2Cfg<KSUB>;
  if (g2_max_pairs<KSUB, EPI>() <= 0) return FDLLM_ERR_CUDA;  // also sets the shared-memory attribute
  // the kernel's __cluster_dims__ gives the pairs; no cluster attribute here
  const cudaError_t e =
      p.sk_tiles < p.tiles
          ? launch_ex(gemm_sk2_kernel<KSUB, EPI, true>, dim3(grid), dim3(kGThreads), C::kSmem, stream, 1,
                      pdl_enabled(), ma, mb0, mb1, mb2, p)
          : launch_ex(gemm_sk2_kernel<KSUB, EPI, false>, dim3(grid), dim3(kGThreads), C::kSmem, stream, 1,
                      pdl_enabled(), ma, mb0, mb1, mb2, p);
  if (e != cudaSuccess) return FDLLM_ERR_CUDA;
  return cudaPeekAtLastError() == cudaSuccess ? FDLLM_OK : FDLLM_ERR_CUDA;
}

template <int EPI>
int dispatch_gemm(const GemmPlan& pl, const CUtensorMap& ma, const CUtensorMap& mb0, const CUtensorMap& mb1,
                  const CUtensorMap& mb2, const GemmParams& p, cudaStream_t stream) {
  if (pl.pair)
    return pl.ksub == 2 ? launch_gemm2_cfg<2, EPI>(ma, mb0, mb1, mb2, p, pl.grid, stream)
                        : launch_gemm2_cfg<1, EPI>(ma, mb0, mb1, mb2, p, pl.grid, stream);
  if (pl.bn == 256) {
    if (pl.xrows == 64)
      return pl.ksub == 2 ? launch_gemm_cfg<256, 64, 2, EPI>(ma, mb0, mb1, mb2, p, pl.grid, stream)
                          : launch_gemm_cfg<256, 64, 1, EPI>(ma, mb0, mb1, mb2, p, pl.grid, stream);
    return launch_gemm_cfg<256, 128, 1, EPI>(ma, mb0, mb1, mb2, p, pl.grid, stream);
  }
  if (pl.xrows == 64)
    return pl.ksub == 2 ? launch_gemm_cfg<128, 64, 2, EPI>(ma, mb0, mb1, mb2, p, pl.grid, stream)
                        : launch_gemm_cfg<128, 64, 1, EPI>(ma, mb0, mb1, mb2, p, pl.grid, stream);
  return pl.ksub == 2 ? launch_gemm_cfg<128, 128, 2, EPI>(ma, mb0, mb1, mb2, p, pl.grid, stream)
                      : launch_gemm_cfg<128, 128, 1, EPI>(ma, mb0, mb1, mb2, p, pl.grid, stream);
}

// Shared set-up: plan, workspace split, tensor maps of A and of the weights.
int run_gemm(int epi, const void* a, int64_t lda, const void* const* w, int n_w, int64_t w_rows, int32_t n_rows,
             int32_t n_cols, int32_t k_dim, GemmParams& p, void* workspace, size_t workspace_bytes,
             cudaStream_t stream) {
  const GemmPlan pl = plan_gemm(epi, n_rows, n_cols, k_dim, p.d_model);
  if (pl.iters < 0 || pl.tiles <= 0 || pl.grid <= 0) return FDLLM_ERR_ARG;
  if (workspace == nullptr || workspace_bytes < gemm_ws_bytes(pl) || !aligned16(workspace))
    return FDLLM_ERR_WORKSPACE;
  p.groups = pl.groups;
  p.n_rows = n_rows;
  p.n_cols = n_cols;
  p.m_tiles = pl.m_tiles;
  p.n_tiles = pl.n_tiles;
  p.kbt = pl.kbt;
  p.iters = pl.iters;
  p.sk_tiles = pl.sk_tiles;
  p.tiles = pl.tiles;
  p.epi = epi;
  p.flags = static_cast<int32_t*>(workspace);
  p.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kGFlagBytes);
  p.status = status_ptr();
  CUtensorMap ma, mb[3];
  int rc;
  if ((rc = make_tmap_bf16_sw128(&ma, a, n_rows, k_dim, lda, pl.xrows)) != FDLLM_OK) return rc;
  // B box: the rows one CTA loads per operand box
  const uint32_t box = pl.pair ? kGBM : (epi == kEpiSwiglu ? pl.bn / 2 : pl.bn);
  for (int i = 0; i < n_w; ++i)
    if ((rc = make_tmap_bf16_sw128(&mb[i], w[i], w_rows, k_dim, k_dim, box)) != FDLLM_OK) return rc;
  for (int i = n_w; i < 3; ++i) mb[i] = mb[0];
  if (epi == kEpiQkv) return dispatch_gemm<kEpiQkv>(pl, ma, mb[0], mb[1], mb[2], p, stream);
  if (epi == kEpiStore) return dispatch_gemm<kEpiStore>(pl, ma, mb[0], mb[1], mb[2], p, stream);
  return dispatch_gemm<kEpiSwiglu>(pl, ma, mb[0], mb[1], mb[2], p, stream);
}

}  // namespace

// QKV through the stream-K kernel (called by the QKV entry points).
int launch_qkv_sk(const void* xn, const void* wq, const void* wk, const void* wv, const int64_t* pos,
                  const float* rope_sin, const float* rope_cos, void* q_out, void* k_out, void* v_out, int32_t n_rows,
                  int32_t d_model, int32_t n_heads, int64_t n_slots, void* workspace, size_t workspace_bytes,
                  int kv_by_slot, cudaStream_t stream) {
  if (n_rows < 0 || n_heads <= 0 || d_model != n_heads * 128 || n_slots <= 0 || d_model % kGBK != 0)
    return FDLLM_ERR_ARG;
  if (n_rows == 0) return FDLLM_OK;
  const void* ptrs[] = {xn, wq, wk, wv, pos, rope_sin, rope_cos, q_out, k_out, v_out};
  for (const void* x : ptrs)
    if (x == nullptr || !aligned16(x)) return FDLLM_ERR_ARG;
  GemmParams p{};
  p.d_model = d_model;
  p.kv_by_slot = kv_by_slot;
  p.n_slots = n_slots;
  p.out0 = static_cast<__nv_bfloat16*>(q_out);
  p.out1 = static_cast<__nv_bfloat16*>(k_out);
  p.out2 = static_cast<__nv_bfloat16*>(v_out);
  p.pos = pos;
  p.sin = rope_sin;
  p.cos = rope_cos;
  const void* w[3] = {wq, wk, wv};
  return run_gemm(kEpiQkv, xn, d_model, w, 3, d_model, n_rows, 3 * d_model, d_model, p, workspace, workspace_bytes,
                  stream);
}

size_t qkv_sk_ws_bytes(int32_t n_rows, int32_t d_model) {
  return gemm_ws_bytes(plan_gemm(kEpiQkv, n_rows, 3 * d_model, d_model, d_model));
}

}  // namespace fdllm

extern "C" {

int fdllm_gemm_set_plan(int32_t bn, int32_t ksub, int32_t grid, int32_t pair, int32_t dp) {
  if ((bn != 0 && bn != 128 && bn != 256) || (ksub != 0 && ksub != 1 && ksub != 2) || grid < 0 || grid > 1024 ||
      pair < -1 || pair > 1 || dp < 0 || dp > 2)
    return FDLLM_ERR_ARG;
  fdllm::GemmOverride& o = fdllm::gemm_override();
  o.bn = bn;
  o.ksub = ksub;
  o.grid = grid;
  o.pair = pair;
  o.dp = dp;
  return FDLLM_OK;
}

size_t fdllm_gemm_workspace_bytes(int32_t n_rows, int32_t n_cols, int32_t k_dim, int32_t swiglu) {
  if (n_rows <= 0 || n_cols <= 0 || k_dim <= 0) return fdllm::kGFlagBytes;
  return fdllm::gemm_ws_bytes(
      fdllm::plan_gemm(swiglu ? fdllm::kEpiSwiglu : fdllm::kEpiStore, n_rows, n_cols, k_dim, 0));
}

int fdllm_gemm_bf16(const void* a, const void* w, void* out, const void* residual, int32_t n_rows, int32_t n_cols,
                    int32_t k_dim, int64_t ld_out, int64_t ld_res, void* workspace, size_t workspace_bytes,
                    cudaStream_t stream) {
  using namespace fdllm;
  if (n_rows < 0 || n_cols <= 0 || k_dim <= 0 || n_cols % 32 != 0 || k_dim % kGBK != 0 || ld_out < n_cols ||
      ld_out % 8 != 0 || (residual != nullptr && (ld_res < n_cols || ld_res % 8 != 0)))
    return FDLLM_ERR_ARG;
  if (n_rows == 0) return FDLLM_OK;
  if (a == nullptr || w == nullptr || out == nullptr || !aligned16(a) || !aligned16(w) || !aligned16(out) ||
      (residual != nullptr && !aligned16(residual)))
    return FDLLM_ERR_ARG;
  GemmParams p{};
  p.out0 = static_cast<__nv_bfloat16*>(out);
  p.res = static_cast<const __nv_bfloat16*>(residual);
  p.ld_out = ld_out;
  p.ld_res = ld_res;
  const void* ws[1] = {w};
  return run_gemm(kEpiStore, a, k_dim, ws, 1, n_cols, n_rows, n_cols, k_dim, p, workspace, workspace_bytes, stream);
}

int fdllm_gemm_swiglu(const void* a, const void* w_gate_up, void* out, int32_t n_rows, int32_t hidden, int32_t k_dim,
                      int64_t ld_out, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  using namespace fdllm;
  if (n_rows < 0 || hidden <= 0 || k_dim <= 0 || hidden % 128 != 0 || k_dim % kGBK != 0 || ld_out < hidden ||
      ld_out % 8 != 0)
    return FDLLM_ERR_ARG;
  if (n_rows == 0) return FDLLM_OK;
  if (a == nullptr || w_gate_up == nullptr || out == nullptr || !aligned16(a) || !aligned16(w_gate_up) ||
      !aligned16(out))
    return FDLLM_ERR_ARG;
  GemmParams p{};
  p.out0 = static_cast<__nv_bfloat16*>(out);
  p.ld_out = ld_out;
  p.hidden = hidden;
  const void* ws[1] = {w_gate_up};
  return run_gemm(kEpiSwiglu, a, k_dim, ws, 1, 2 * hidden, n_rows, 2 * hidden, k_dim, p, workspace, workspace_bytes,
                  stream);
}

}  // extern "C"
