// Recompute attention on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
// Same contract as the CUDA-core path in attn_rows.cu (tread/blend.py:76,110 and the query
// forward of tread/engine.py:131-132): row r of head h attends to every cache key at a position
// <= pos[r] of KV head h / (Hq/Hkv). This path covers bf16/fp16 with head_dim 128.
//
// Work items and schedules. An item is a tile of 128 consecutive rows of one query head; it takes
// n = (latest position among its rows) / 128 + 1 key blocks ("steps"). A CTA runs its pieces (an
// item's whole key range or a contiguous part of it) one after another.
//   - tail split (default with a workspace): one CTA per SM; full rounds of whole items, longest
//     first, in snake order, then the items left over split by key range over all CTAs (the
//     split cap chosen by an estimate of every CTA's finish; details at the plan below);
//   - stream-K (on request): all items' steps laid end to end (items of one KV head together, for
//     L2 reuse of its K/V) and cut into one equal contiguous segment per CTA;
//   - whole tiles (no workspace): one CTA per item, latest rows first.
// An item cut between CTAs leaves partial results (unnormalised O, running max m and sum l per
// row) in the workspace; after its last piece a CTA counts its (at most two) partial pieces in,
// and the one that completes an item (an atomic count per item, no waiting) merges its partials,
// bulk-copied into its idle tile buffers:
//     O = sum_k O_k 2^(m_k - M) / sum_k l_k 2^(m_k - M),  M = max_k m_k.
//
// Roles and pipeline per CTA:
//   - loader (lane 0 of warp 9): TMA (128-byte swizzle) loads each piece's Q tile and 128-key K
//     and V tiles into separate 2-stage rings, refilling a stage when the MMA that read it commits
//     to that stage's "free" barrier; the next piece's Q loads once the last QK of the current
//     piece has read the old one;
//   - MMA issuer (warp 8; descriptors warp-uniform, one elected lane issues): S_g = Q K_g^T
//     (8 x tcgen05.mma kind::f16, M=N=K=128, operands in shared memory) into TMEM S buffer g%2, so
//     QK(g+1) runs while the rows are in the softmax of step g, and PV_g as two K=64 halves,
//     O_h += P_g[:, half h] V_g[half h, :], with P read from TMEM;
//   - softmax (warps 0-7; a row = a TMEM lane, its 128 key columns split into two halves, one per
//     warp): reads its half of S once, masks keys past the row's position, keeps the half's own
//     running max and sum in the exp2 domain (ex2.approx on the MUFU, a share of the pairs as a
//     cubic on the FMA pipe), rescales the half's O in TMEM
//     only when its max grows by more than 8 (a stale max is exact since 1/l uses the same max; a
//     warp decides together because tcgen05.ld/st are warp-collective), and writes P over the S
//     columns it has just read. The halves are merged once per piece, in the epilogue.
// Steps are counted across a CTA's pieces, so the barrier phases (one barrier per S buffer and
// ring stage: a parity wait never aliases) run on unchanged. TMEM: S buffers at columns 0 and
// 128, the key halves' O accumulators at 256 and 384 (512 allocated; one CTA per SM). Every wait
// is bounded in wall time and aborts the CTA through a shared flag; an aborted CTA records bit 2
// in *err, lets issued copies and MMAs land, frees its TMEM and returns (the workspace's counters
// must then be zeroed before the next call).
#include <cuda.h>

#include <algorithm>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "tcgen05.cuh"

namespace tread {

namespace tc {

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

bool make_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, uint64_t nd, uint64_t ny, uint64_t nz,
              uint64_t sy, uint64_t sz, uint32_t by, uint32_t bz) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {nd, ny, nz};
  const cuuint64_t strides[2] = {sy * 2, sz * 2};
  const cuuint32_t box[3] = {64, by, bz};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace tc

int attn_rows_simt(const void* q, const void* K, const void* V, long long c_sh, long long T_cache, const int64_t* pos,
                   int R, int Hq, int Hkv, int D, float sm_scale, void* out, int dtype, unsigned* err,
                   cudaStream_t st);

namespace {

using namespace tc;

constexpr int kRows = 128;   // query rows per item (MMA M)
constexpr int kKeys = 128;   // keys per step (MMA N of Q K^T, K of P V)
constexpr int kD = 128;      // head_dim (MMA K of Q K^T, N of P V)
constexpr int kBlock = 16384;  // one 128 x 64 16-bit swizzled block
constexpr int kMaxTiles = 2048;  // row tiles the stream-K plan tables hold (shared memory)
// Q 2 buffers, K and V rings 2 stages, 2 blocks each (a buffer of Q lets the next piece's tile load
// while the current piece runs)
constexpr int kTilesBytes = 12 * kBlock;
constexpr int kSmem = 1024 + kTilesBytes + 8 * kMaxTiles + 512;
// Stream-K cost of an item's start and end (pipeline fill and drain, epilogue), in steps.
constexpr int kPieceCost = 3;
// Exponentials per 16 keys of a softmax lane computed as a polynomial on the FMA pipe instead of
// ex2 on the MUFU (in pairs). Measured on B200, 2 of every 8 pairs is fastest: the softmax step is
// latency-bound, and the polynomial shortens its chains of dependent exponentials.
#ifndef TREAD_ATTN_POLY_PAIRS
#define TREAD_ATTN_POLY_PAIRS 2
#endif
constexpr int kPolyPairs = TREAD_ATTN_POLY_PAIRS;
constexpr int kTailSplit = 8;  // most key ranges one tail-round tile is split into
constexpr int kMergeCost = 3;  // units charged to a split part for its partial store and merge
// TMEM columns: S buffers 0-127 and 128-255 (fp32; each column half also holds that half's P,
// 16-bit pairs, once read), O accumulators of key halves 0 and 1 at 256-383 and 384-511.
constexpr uint32_t kTmemO = 256;
// workspace: one arrival counter per item (at most kMaxItems), then 2 partial slots per CTA:
// O [128][128] fp32, m [128], l [128]
constexpr int kMaxItems = 1 << 16;
constexpr size_t kCounterBytes = (size_t)kMaxItems * 4;
constexpr size_t kSlotBytes = (size_t)kRows * kD * 4 + 2 * kRows * 4;

// Warps 0-7 run the softmax: warp w covers TMEM lanes (rows) 32*(w%4).. and S columns 64*(w/4)..
// of its row quadrant; warp 8 issues every tcgen05.mma; lane 0 of warp 9 every TMA load.
constexpr int kWarpsPerQuad = 2;
constexpr int kSoftWarps = 4 * kWarpsPerQuad;
constexpr int kColsPerWarp = kKeys / kWarpsPerQuad;  // 64
constexpr int kMmaWarp = kSoftWarps, kLoadWarp = kSoftWarps + 1;
constexpr int kThreadsTC = (kSoftWarps + 2) * 32;


// Item p -> (query head, row tile): items of one KV group together, tile by tile, head by head.
struct Item {
  int head, tile, kvh;
};
__device__ __forceinline__ Item item_of(int p, int G, int ntiles) {
  const int per_group = G * ntiles;
  const int g = p / per_group, r = p - g * per_group;
  const int t = r / G;
  return Item{g * G + (r - t * G), t, g};
}

// Schedules: kWhole, one CTA per tile, latest rows first; kStreamK, equal shares of all tiles' key
// blocks per CTA; kTail, persistent CTAs running whole tiles latest first, the tiles left after the
// full rounds split into key ranges over the CTAs.
enum { kWhole = 0, kStreamK = 1, kTail = 2 };

struct Piece {
  int item, j0, j1, n_item;
  bool first;  // stream-K: first piece of this CTA's segment (workspace slot 2c, else 2c+1)
};

// Stream-K segments: CTA c owns units [seg(c), seg(c+1)) of the U units laid end to end in item
// order. Item p costs its steps (units [start, start + steps), real key blocks) plus kPieceCost
// trailing units for its start and end, so a CTA given many short items is given fewer steps;
// a segment boundary inside those trailing units cuts nothing. All G heads of a row tile take the
// tile's steps ts[t], so the layout has a closed form over tc[], the tiles' inclusive prefix of
// (ts + kPieceCost): a KV group spans UG = G * tc[ntiles-1] units and item (g, t, hh) starts at
// g * UG + G * tc[t-1] + hh * (ts[t] + kPieceCost).
struct Plan {
  const int* ts;
  const int* tc;
  int G, ntiles;
  long long UG, U;
  int grid;
  __device__ __forceinline__ long long seg(int c) const { return (long long)c * U / grid; }
  __device__ __forceinline__ int steps(int p) const { return ts[(p % (G * ntiles)) / G]; }
  __device__ __forceinline__ long long start_of(int p) const {
    const int g = p / (G * ntiles), r = p - g * G * ntiles, t = r / G, hh = r - t * G;
    return g * UG + (long long)G * (t ? tc[t - 1] : 0) + (long long)hh * (ts[t] + kPieceCost);
  }
  __device__ __forceinline__ int item_at(long long u) const {  // the item whose units hold unit u
    const int g = (int)(u / UG);
    const long long r = u - g * UG;
    int lo = 0, hi = ntiles - 1;  // first tile t with G * tc[t] > r
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if ((long long)G * tc[mid] > r) hi = mid; else lo = mid + 1;
    }
    const int hh = (int)((r - (long long)G * (lo ? tc[lo - 1] : 0)) / (ts[lo] + kPieceCost));
    return g * G * ntiles + lo * G + hh;
  }
  __device__ __forceinline__ int cta_of(long long u) const {  // the CTA whose segment holds unit u
    int c = (int)((u * grid) / U);
    while (c + 1 < grid && seg(c + 1) <= u) ++c;
    while (c > 0 && seg(c) > u) --c;
    return c;
  }
  // workspace slot of item p's piece in CTA cx: 2cx if it is the first real piece of cx's segment
  // (no earlier item's real steps in it), else 2cx + 1
  __device__ __forceinline__ int slot_of(int p, int cx) const {
    return 2 * cx + ((p == 0 || seg(cx) >= start_of(p) - kPieceCost) ? 0 : 1);
  }
};

__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

template <typename T>
__global__ void __launch_bounds__(kThreadsTC, 1)
    attn_rows_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const int64_t* __restrict__ pos, int R, int Hq,
                        int G, long long T_cache, float scale_log2, T* __restrict__ out, unsigned* err,
                        unsigned char* __restrict__ ws, int mode) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sQ = smem;               // 2 buffers x 2 blocks (d 0-63, d 64-127)
  unsigned char* sK = smem + 4 * kBlock;  // 2 stages x 2 blocks
  unsigned char* sV = smem + 8 * kBlock;  // 2 stages x 2 blocks
  int* s_tsteps = reinterpret_cast<int*>(smem + kTilesBytes);  // [tile] steps
  int* s_tpre = s_tsteps + kMaxTiles;  // [tile] inclusive prefix of steps + kPieceCost
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_tpre + kMaxTiles);
  uint64_t* q_full = bars + 0;   // [2] Q buffer loaded
  uint64_t* k_full = bars + 2;   // [2] K stage loaded
  uint64_t* v_full = bars + 4;   // [2] V stage loaded
  uint64_t* s_full = bars + 6;   // [2] S buffer written by QK
  uint64_t* q_free = bars + 8;   // [2] Q buffer read by its piece's last QK
  uint64_t* o_free = bars + 10;  // O read by the piece's epilogue (256 arrivals)
  uint64_t* p_full = bars + 11;  // [2] P of S buffer b written by the softmax (256 arrivals)
  uint64_t* pv_done = bars + 13; // [2] PV of S buffer b's P complete (buffer reusable, O stable)
  uint64_t* k_free = bars + 15;  // [2] K stage read by its QK
  uint64_t* v_free = bars + 17;  // [2] V stage read by its PV
  uint64_t* quad_bar = bars + 19; // [4] the two softmax warps of a row quadrant (64 arrivals)
  uint64_t* soft_bar = bars + 23; // all softmax warps (256 arrivals)
  uint64_t* bulk_bar = bars + 24; // merge: partial slots copied into shared memory
  constexpr int kNumBars = 25;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + kNumBars);
  int* s_abort = reinterpret_cast<int*>(bars + kNumBars + 1);
  int* s_merge = s_abort + 1;  // [2] merge decisions of this CTA's (at most two) partial pieces
  int* s_fin = s_abort + 4;    // [4] kTail: latest estimated CTA finish under split caps 1, 2, 4, 8
  __shared__ float s_part[2][kWarpsPerQuad][kRows];  // [max / sum][key half][row]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ntiles = (R + kRows - 1) / kRows;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(s_tmem)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 32) {
    for (int i = 0; i < kNumBars; ++i) mbar_init(bars + i, 1);
    mbar_init(o_free, kSoftWarps * 32);
    mbar_init(&p_full[0], kSoftWarps * 32);
    mbar_init(&p_full[1], kSoftWarps * 32);
    for (int i = 0; i < 4; ++i) mbar_init(&quad_bar[i], kWarpsPerQuad * 32);
    mbar_init(soft_bar, kSoftWarps * 32);
    *s_abort = 0;
    for (int i = 0; i < 4; ++i) s_fin[i] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }

  // ---- steps of a row tile (one warp: the latest valid position among its rows)
  auto tile_steps = [&](int t) -> int {
    long long mx = 0;
#pragma unroll
    for (int k = 0; k < kRows / 32; ++k) {
      const int r = t * kRows + k * 32 + lane;
      if (r < R) {
        const long long p = pos[r];
        if (p >= 0 && p < T_cache) mx = p > mx ? p : mx;
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const long long y = __shfl_xor_sync(0xffffffffu, mx, o);
      mx = y > mx ? y : mx;
    }
    return (int)(mx / kKeys) + 1;
  };
  const bool stream_k = mode == kStreamK;
  if (mode != kWhole) {
    // all tiles, one warp each (tiles warp, warp + 10, ...), eight tiles' position loads in flight
    // together before their reductions
    constexpr int kWarps = kThreadsTC / 32;
    for (int t0 = warp; t0 < ntiles; t0 += 8 * kWarps) {
      long long p[8][kRows / 32];
#pragma unroll
      for (int k = 0; k < 8; ++k)
#pragma unroll
        for (int j = 0; j < kRows / 32; ++j) {
          const int r = (t0 + k * kWarps) * kRows + j * 32 + lane;
          p[k][j] = t0 + k * kWarps < ntiles && r < R ? pos[r] : -1;
        }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int t = t0 + k * kWarps;
        if (t >= ntiles) break;  // warp-uniform
        long long mx = 0;
#pragma unroll
        for (int j = 0; j < kRows / 32; ++j)
          if (p[k][j] >= 0 && p[k][j] < T_cache) mx = p[k][j] > mx ? p[k][j] : mx;
#pragma unroll
        for (int o = 16; o; o >>= 1) {
          const long long y = __shfl_xor_sync(0xffffffffu, mx, o);
          mx = y > mx ? y : mx;
        }
        if (lane == 0) s_tsteps[t] = (int)(mx / kKeys) + 1;
      }
    }
    __syncthreads();
    if (stream_k && warp == 0) {  // inclusive prefix of the tiles' steps
      int carry = 0;
      for (int base = 0; base < ntiles; base += 32) {
        const int t = base + lane;
        int v = t < ntiles ? s_tsteps[t] + kPieceCost : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, v, o);
          if (lane >= o) v += y;
        }
        if (t < ntiles) s_tpre[t] = carry + v;
        carry += __shfl_sync(0xffffffffu, v, 31);
      }
    }
  } else if (warp == 0) {
    const int st = tile_steps(ntiles - 1 - (int)blockIdx.x / Hq);
    if (lane == 0) s_tsteps[0] = st;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  const long long UG = stream_k ? (long long)G * s_tpre[ntiles - 1] : 0;  // units of one KV group
  const Plan plan{s_tsteps, s_tpre, G, ntiles, UG, UG * (Hq / G), (int)gridDim.x};
  const int c = blockIdx.x;
  long long cur = stream_k ? plan.seg(c) : 0;
  const long long seg_end = stream_k ? plan.seg(c + 1) : 1;
  // kWhole / kTail items are encoded -1 - i, i the position in the latest-first list (head i % Hq,
  // row tile ntiles - 1 - i / Hq), so items run longest first. kTail: S CTAs take F full rounds in
  // snake order (round k gives item k*S + c, or k*S + S-1 - c for odd k, pairing long with short).
  // The r items left are split over the S CTAs by their rank in the tail round (c for even F,
  // S-1 - c for odd): item F*S + q gets w_q = S/r key ranges, one more for the S % r longest items
  // (q < S % r), at most a cap W; part p (of n steps) is steps [p*n/w_q, (p+1)*n/w_q) on rank
  // first(q) + p, first(q) = q*w + min(q, S % r). Empty parts are skipped. W is the one of 1, 2, 4,
  // 8 (kTailSplit) whose estimated latest CTA finish (full-round units + the CTA's tail part, a split
  // part also paying kMergeCost) is lowest; W = 1 runs the tail items whole on the lightest CTAs.
  // Without full rounds every CTA is idle and W = kTailSplit.
  const int nitems = Hq * ntiles;
  const int tS = (int)gridDim.x, tF = nitems / tS, tR = nitems - tF * tS;
  auto split_of = [&](int W, int& w, int& x) {  // parts per tail item under cap W: w, +1 for q < x
    w = tS / tR;
    x = tS - w * tR;
    if (w >= W) w = W, x = 0;
  };
  int tW = 1, tX = 0;
  if (mode == kTail && tR > 0) {
    int cap = kTailSplit;
    if (tF > 0) {
      // a / b for the small non-negative operands here (< 2^22): float reciprocal, then one
      // correction step (integer division by a runtime value is a long dependent sequence)
      auto fdiv = [](int a, int b, float inv_b) {
        int d = (int)((float)a * inv_b);
        d += (d + 1) * b <= a;
        d -= d * b > a;
        return d;
      };
      const float inv_hq = 1.f / (float)Hq;
      auto div_hq = [&](int i) { return fdiv(i, Hq, inv_hq); };
      // full-round units of every CTA (into the stream-K prefix table, unused by kTail)
      for (int cx = tid; cx < tS; cx += kThreadsTC) {
        int L = 0;
        for (int k = 0; k < tF; ++k)
          L += s_tsteps[ntiles - 1 - div_hq(k * tS + ((k & 1) ? tS - 1 - cx : cx))] + kPieceCost;
        s_tpre[cx] = L;
      }
      __syncthreads();
      // warps 2e and 2e + 1 estimate every CTA's finish under cap 2^e; one shared atomic per warp
      if (warp < 8) {
        const int e = warp >> 1;
        int w, x;
        split_of(1 << e, w, x);
        const int hi = x * (w + 1);
        const float inv_w = 1.f / (float)w, inv_w1 = 1.f / (float)(w + 1);
        int fmax = 0;
        for (int cx = (warp & 1) * 32 + lane; cx < tS; cx += 64) {
          const int rk = (tF & 1) ? tS - 1 - cx : cx;
          const int q = rk < hi ? fdiv(rk, w + 1, inv_w1) : x + fdiv(rk - hi, w, inv_w);
          int fin = s_tpre[cx];
          if (q < tR) {
            const bool big = q < x;
            const int wq = big ? w + 1 : w, p = rk - (q * w + min(q, x));
            const float inv_wq = big ? inv_w1 : inv_w;
            const int n = s_tsteps[ntiles - 1 - div_hq(tF * tS + q)];
            const int part = fdiv((p + 1) * n, wq, inv_wq) - fdiv(p * n, wq, inv_wq);
            if (part > 0) fin += part + kPieceCost + (part < n ? kMergeCost : 0);
          }
          fmax = max(fmax, fin);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) fmax = max(fmax, __shfl_xor_sync(0xffffffffu, fmax, o));
        if (lane == 0) atomicMax(&s_fin[e], fmax);
      }
      __syncthreads();
      cap = 1;
      for (int e = 1; e < 4; ++e)
        if (s_fin[e] < s_fin[__ffs(cap) - 1]) cap = 1 << e;
    }
    split_of(cap, tW, tX);
  }
  auto part_first = [&](int q) { return q * tW + min(q, tX); };
  auto nparts = [&](int q) { return tW + (q < tX ? 1 : 0); };
  const int trank = (tF & 1) ? tS - 1 - c : c;  // this CTA's rank in the tail round
  int tk = 0;  // kTail: index of this CTA's current piece
  auto tail_piece = [&](Piece& pc) -> bool {
    while (true) {
      int i, p = 0, w = 1;
      if (tk < tF) {
        i = tk * tS + ((tk & 1) ? tS - 1 - c : c);
      } else if (tk == tF) {
        const int hi = tX * (tW + 1);
        const int q = trank < hi ? trank / (tW + 1) : tX + (trank - hi) / tW;
        if (q >= tR) return false;
        p = trank - part_first(q);
        w = nparts(q);
        i = tF * tS + q;
      } else {
        return false;
      }
      ++tk;
      const int n = s_tsteps[ntiles - 1 - i / Hq];
      int j0 = 0, j1 = n;
      if (i >= tF * tS) {
        j0 = p * n / w;
        j1 = (p + 1) * n / w;
        if (j0 == j1) continue;  // fewer steps than parts
      }
      pc.item = -1 - i;
      pc.n_item = n;
      pc.j0 = j0;
      pc.j1 = j1;
      pc.first = false;
      return true;
    }
  };
  // this CTA's pieces, in order
  auto first_piece = [&](Piece& pc) -> bool {
    if (mode == kWhole) {  // one whole tile: latest rows first
      pc.item = -1 - c;
      pc.n_item = s_tsteps[0];
      pc.j0 = 0;
      pc.j1 = pc.n_item;
      pc.first = true;
      return true;
    }
    if (mode == kTail) return tail_piece(pc);
    if (cur >= seg_end) return false;
    pc.item = plan.item_at(cur);
    long long u0 = plan.start_of(pc.item);
    pc.n_item = plan.steps(pc.item);
    if (cur - u0 >= pc.n_item) {  // the segment starts in an item's trailing cost units
      u0 += pc.n_item + kPieceCost;
      if (u0 >= seg_end) return false;
      pc.item += 1;
      pc.n_item = plan.steps(pc.item);
      cur = u0;
    }
    pc.j0 = (int)(cur - u0);
    pc.j1 = (int)(min(seg_end - u0, (long long)pc.n_item));
    pc.first = true;
    return true;
  };
  auto next_piece = [&](Piece& pc) -> bool {
    if (mode == kTail) return tail_piece(pc);
    if (!stream_k) return false;
    const long long u1 = plan.start_of(pc.item) + pc.n_item + kPieceCost;  // the next item's start
    if (u1 >= seg_end) return false;
    pc.item += 1;
    pc.n_item = plan.steps(pc.item);
    pc.j0 = 0;
    pc.j1 = (int)(min(seg_end - u1, (long long)pc.n_item));
    pc.first = false;
    return true;
  };
  auto item_coords = [&](const Piece& pc) -> Item {
    if (pc.item < 0) {
      const int cc = -1 - pc.item;
      const int h = cc % Hq;
      return Item{h, ntiles - 1 - cc / Hq, h / G};
    }
    return item_of(pc.item, G, ntiles);
  };
  const Waiter wait{s_abort};

  if (warp == kLoadWarp) {
    // ------------------------------------------------------------------ TMA loader (one lane)
    // K and V have separate 2-stage rings; K(g+2) goes into its stage once QK(g) has read it and
    // V(g+2) once PV(g) has, so copies run two steps ahead of the MMAs.
    if (lane == 0) {
      Piece pc;
      int k = 0;
      long long g = 0;
      bool ok = true;
      for (bool more = first_piece(pc); more && ok; more = next_piece(pc), ++k) {
        const Item it = item_coords(pc);
        const int qb = k & 1;
        if (k >= 2 && !(ok = wait(&q_free[qb], ((k - 2) >> 1) & 1))) break;
        mbar_expect_tx(&q_full[qb], 2 * kBlock);
        tma_load_3d(sQ + qb * 2 * kBlock, &tm_q, &q_full[qb], 0, it.head, it.tile * kRows);
        tma_load_3d(sQ + qb * 2 * kBlock + kBlock, &tm_q, &q_full[qb], 64, it.head, it.tile * kRows);
        for (int j = pc.j0; j < pc.j1; ++j, ++g) {
          const int s = (int)(g & 1);
          const uint32_t ph = (uint32_t)(((g - 2) >> 1) & 1);
          if (g >= 2 && !(ok = wait(&k_free[s], ph))) break;
          mbar_expect_tx(&k_full[s], 2 * kBlock);
          tma_load_3d(sK + s * 2 * kBlock, &tm_k, &k_full[s], 0, j * kKeys, it.kvh);
          tma_load_3d(sK + s * 2 * kBlock + kBlock, &tm_k, &k_full[s], 64, j * kKeys, it.kvh);
          if (g >= 2 && !(ok = wait(&v_free[s], ph))) break;
          mbar_expect_tx(&v_full[s], 2 * kBlock);
          tma_load_3d(sV + s * 2 * kBlock, &tm_v, &v_full[s], 0, j * kKeys, it.kvh);
          tma_load_3d(sV + s * 2 * kBlock + kBlock, &tm_v, &v_full[s], 64, j * kKeys, it.kvh);
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------ MMA issuer (one warp)
    constexpr uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
    constexpr uint32_t idesc_qk = idesc_f16(fmt, 0, kRows, kKeys);
    constexpr uint32_t idesc_pv = idesc_f16(fmt, 1, kRows, kD);
    // descriptors of stage 0, chunk 0; stages and chunks add (byte offset >> 4) to the address
    const uint64_t dq = sw128_desc(smem_u32(sQ), 16, 1024), dk0 = sw128_desc(smem_u32(sK), 16, 1024);
    const uint64_t dv0 = sw128_desc(smem_u32(sV), kBlock, 1024);
    constexpr uint64_t kStage = (2 * kBlock) >> 4;
    // PV(g): O_h += P_g[:, keys of half h] V_g[keys of half h, :] for h = 0, 1; P of half h sits in
    // S buffer g%2 at columns 64*h .. 64*h+31 (packed pairs); `fresh` starts each half's O anew
    auto issue_pv = [&](long long g, bool fresh) {
      const int b = (int)(g & 1);
      const uint64_t vb = dv0 + (uint64_t)b * kStage;
#pragma unroll
      for (int h = 0; h < 2; ++h) {  // one group of four per key half
        uint32_t ta[4];
        uint64_t vd[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int kk = 4 * h + i;
          ta[i] = tmem + b * kKeys + h * 64 + i * 8;
          vd[i] = vb + (uint64_t)((kk * 16 * 128) >> 4);
        }
        mma_f16_ts_x4_elect(tmem + kTmemO + h * 128, ta, vd, idesc_pv, fresh ? 0u : 1u);
      }
      mma_commit_elect(&pv_done[b]);
      mma_commit_elect(&v_free[b]);
    };
    // Steps of all pieces in order: QK(g), then PV of the step before (possibly the previous
    // piece's last), so the next piece's first QK goes in before the current piece's last PV and
    // the tensor pipe does not drain at a piece boundary.
    Piece pc;
    int k = 0, pk = 0;
    long long g = 0, pg = -1;  // pg: step whose PV is still to be issued
    bool p_fresh = false, ok = true;
    auto pv_prev = [&]() -> bool {  // PV(pg): its P, its V stage, and (a piece's first PV) O read out
      const int b = (int)(pg & 1);
      if (!__all_sync(0xffffffffu, wait(&p_full[b], (pg >> 1) & 1) && wait(&v_full[b], (pg >> 1) & 1) &&
                                       (!p_fresh || pk == 0 || wait(o_free, (pk - 1) & 1))))
        return false;
      tc_fence_after();
      issue_pv(pg, p_fresh);
      return true;
    };
    for (bool more = first_piece(pc); more && ok; more = next_piece(pc), ++k) {
      const int n = pc.j1 - pc.j0;
      const int qb = k & 1;
      const uint64_t dqk = dq + (uint64_t)qb * kStage;
      for (int jl = 0; jl < n && ok; ++jl, ++g) {
        const int s = (int)(g & 1);
        // S buffer s holds P(g-2) until PV(g-2) has read it
        ok = __all_sync(0xffffffffu, wait(&k_full[s], (g >> 1) & 1) &&
                                         (jl > 0 || wait(&q_full[qb], (k >> 1) & 1)) &&
                                         (g < 2 || wait(&pv_done[s], ((g - 2) >> 1) & 1)));
        if (!ok) break;
        tc_fence_after();
        const uint64_t kb = dk0 + (uint64_t)s * kStage;
        {
          uint64_t ad[8], bd[8];
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk) {
            const uint64_t off = (uint64_t)(((kk >> 2) * kBlock + (kk & 3) * 32) >> 4);
            ad[kk] = dqk + off;
            bd[kk] = kb + off;
          }
          mma_f16_x8_elect(tmem + s * kKeys, ad, bd, idesc_qk, 0u);
        }
        mma_commit_elect(&s_full[s]);
        mma_commit_elect(&k_free[s]);
        if (jl == n - 1) mma_commit_elect(&q_free[qb]);
        if (pg >= 0 && !(ok = pv_prev())) break;
        pg = g;
        p_fresh = jl == 0;
        pk = k;
      }
    }
    if (ok && pg >= 0) pv_prev();
  } else {
    // ------------------------------------------------------------------ softmax
    // Each key half keeps its own running max, sum and O accumulator, so the two warps of a lane
    // quadrant never wait for each other; the halves are merged once per piece, in the epilogue.
    const int quad = warp & 3, part = warp >> 2;
    const int trow = quad * 32 + lane;  // row within the tile (= TMEM lane)
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t col = part * kColsPerWarp;
    const uint32_t tOh = tmem + kTmemO + part * 128;  // this half's O accumulator
    unsigned* counters = reinterpret_cast<unsigned*>(ws);
    unsigned char* slots = ws ? ws + kCounterBytes : nullptr;
    // bounded barriers among softmax warps (an aborting warp never strands a partner): arrive,
    // then wait for the phase this thread's own count says is next
    uint32_t quad_phase = 0, soft_phase = 0, bulk_phase = 0;
    auto quad_sync = [&]() -> bool {
      mbar_arrive(&quad_bar[quad]);
      return __all_sync(0xffffffffu, wait(&quad_bar[quad], (quad_phase++) & 1));
    };
    auto soft_sync = [&]() -> bool {
      mbar_arrive(soft_bar);
      return __all_sync(0xffffffffu, wait(soft_bar, (soft_phase++) & 1));
    };
    Piece pc, partials[2];
    int k = 0, npart = 0;
    long long g = 0;
    bool ok = true;
    for (bool more = first_piece(pc); more && ok; more = next_piece(pc), ++k) {
      const Item it = item_coords(pc);
      const int row = it.tile * kRows + trow;
      const bool live = row < R;
      long long p = live ? pos[row] : 0;
      if (live && (p < 0 || p >= T_cache)) {
        if (part == 0 && err) atomicOr(err, 2u);
        p = 0;
      }
      // padding rows past R (output discarded) see every key, so they never take the masking path
      if (!live) p = (long long)pc.n_item * kKeys - 1;
      float m = -INFINITY, l = 0.f;
      const int n = pc.j1 - pc.j0;
      for (int jl = 0; jl < n; ++jl, ++g) {
        const int s = (int)(g & 1);
        ok = __all_sync(0xffffffffu, wait(&s_full[s], (g >> 1) & 1));
        if (!ok) break;
        tc_fence_after();
        float v[kColsPerWarp];
        {
          uint32_t r[kColsPerWarp / 32][32];
#pragma unroll
          for (int cc = 0; cc < kColsPerWarp / 32; ++cc)
            tmem_ld32_async(tmem + s * kKeys + col + cc * 32 + lane_off, r[cc]);
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
          for (int cc = 0; cc < kColsPerWarp / 32; ++cc)
#pragma unroll
            for (int i = 0; i < 32; ++i) v[cc * 32 + i] = __uint_as_float(r[cc][i]);
        }
        const long long key0 = (long long)(pc.j0 + jl) * kKeys + col;
        if (__any_sync(0xffffffffu, key0 + kColsPerWarp - 1 > p)) {
          // keys i > lim of this half are past the row's position (one 32-bit compare each)
          const int lim = (int)max(-1LL, min((long long)kColsPerWarp, p - key0));
#pragma unroll
          for (int i = 0; i < kColsPerWarp; ++i)
            if (i > lim) v[i] = -INFINITY;
        }
        float m4[4] = {v[0], v[1], v[2], v[3]};  // four independent 3-input max chains
#pragma unroll
        for (int i = 4; i < kColsPerWarp; i += 2) m4[(i >> 1) & 3] = fmax3(m4[(i >> 1) & 3], v[i], v[i + 1]);
        const float tmax = fmax3(m4[0], m4[1], fmaxf(m4[2], m4[3]));
        const float m_new = fmaxf(m, tmax * scale_log2);  // -inf while every key of this half is masked
        const bool rescale = jl > 0 && m_new > m + 8.f;
        float alpha = 1.f;
        if (jl == 0 || rescale) {
          alpha = m == -INFINITY ? 0.f : ex2(m - m_new);
          l *= alpha;
          m = m_new;
        }
        const float mu = m == -INFINITY ? 0.f : m;  // all-masked half: exponentials of -inf give 0
        uint32_t pk[kColsPerWarp / 2];
        const float2 sc2 = make_float2(scale_log2, scale_log2), nm2 = make_float2(-mu, -mu);
        float2 l2 = make_float2(0.f, 0.f);  // even / odd key sums
#pragma unroll
        for (int i = 0; i < kColsPerWarp; i += 2) {
          const float2 x = ffma2(make_float2(v[i], v[i + 1]), sc2, nm2);
          // kPolyPairs of every 8 pairs on the FMA pipe, the rest on the MUFU
          const float2 pp = (i % 16) < 2 * kPolyPairs ? exp2_poly2(x) : make_float2(ex2(x.x), ex2(x.y));
          l2 = fadd2(l2, pp);
          pk[i / 2] = pack2<T>(pp.x, pp.y);
          // the first half of P goes out while the second half is computed
          if (i == kColsPerWarp / 2 - 2) tmem_st16u(tmem + s * kKeys + part * 64 + lane_off, pk);
        }
        l += l2.x + l2.y;
        // this half's O must be stable (PV(g-1) complete) to rescale it; tcgen05.ld/st are
        // warp-collective, so the warp rescales together, other lanes by 1
        if (__any_sync(0xffffffffu, rescale)) {
          ok = __all_sync(0xffffffffu, wait(&pv_done[s ^ 1], ((g - 1) >> 1) & 1));
          if (!ok) break;
          tc_fence_after();
#pragma unroll 1
          for (int cc = 0; cc < kD / 32; ++cc) {
            float o[32];
            tmem_ld32(tOh + lane_off + cc * 32, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st32(tOh + lane_off + cc * 32, o);
          }
        }
        // P over this warp's own S columns (already in registers): QK(g+2) waits for PV(g)
        tmem_st16u(tmem + s * kKeys + part * 64 + 16 + lane_off, pk + 16);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        mbar_arrive(&p_full[s]);
      }
      if (!ok) break;
      // ---- epilogue of the piece: O final once its last PV completed (PV(g-2), on the other
      // buffer, completed before QK(g-1) was issued)
      ok = __all_sync(0xffffffffu, wait(&pv_done[(g - 1) & 1], ((g - 1) >> 1) & 1));
      if (!ok) break;
      tc_fence_after();
      // merge the halves: O = O_0 2^(m_0 - M) + O_1 2^(m_1 - M), l = l_0 2^(m_0 - M) + l_1 2^(m_1 - M)
      s_part[0][part][trow] = m;
      s_part[1][part][trow] = l;
      if (!(ok = quad_sync())) break;
      const float m0 = s_part[0][0][trow], m1 = s_part[0][1][trow];
      const float M = fmaxf(m0, m1);
      const float a0 = m0 == -INFINITY ? 0.f : ex2(m0 - M), a1 = m1 == -INFINITY ? 0.f : ex2(m1 - M);
      const float L = s_part[1][0][trow] * a0 + s_part[1][1][trow] * a1;
      const bool whole = pc.j0 == 0 && pc.j1 == pc.n_item;
      const float c0 = whole ? a0 / L : a0, c1 = whole ? a1 / L : a1;  // whole: L > 0 (key 0 visible)
      T* orow = out + ((long long)row * Hq + it.head) * kD + col;
      // partial slot layout, coalesced for a warp's 32 consecutive rows: O as [32 float4 columns]
      // [128 rows] float4, then m [128], l [128]
      // kTail: a CTA's only partial is its last piece, in slot 2 * rank + 1
      const int my_si = stream_k ? 2 * c + (pc.first ? 0 : 1) : 2 * trank + 1;
      unsigned char* my_slot = whole ? nullptr : slots + (size_t)my_si * kSlotBytes;
      float own[kColsPerWarp];  // the piece's O of the warp's 64 columns (divided by L for a whole tile)
#pragma unroll
      for (int cc = 0; cc < kColsPerWarp / 32; ++cc) {
        float o0[32], o1[32];
        tmem_ld32(tmem + kTmemO + col + lane_off + cc * 32, o0);
        tmem_ld32(tmem + kTmemO + 128 + col + lane_off + cc * 32, o1);
#pragma unroll
        for (int i = 0; i < 32; ++i) own[cc * 32 + i] = fmaf(o0[i], c0, o1[i] * c1);
      }
      tc_fence_before();
      mbar_arrive(o_free);  // O read: the next piece's first PV may overwrite it
      if (whole) {
        if (live) {
#pragma unroll
          for (int i = 0; i < kColsPerWarp; i += 8) {
            uint4 w = make_uint4(pack2<T>(own[i], own[i + 1]), pack2<T>(own[i + 2], own[i + 3]),
                                 pack2<T>(own[i + 4], own[i + 5]), pack2<T>(own[i + 6], own[i + 7]));
            *reinterpret_cast<uint4*>(orow + i) = w;
          }
        }
        if (!(ok = quad_sync())) break;  // s_part is rewritten by the next piece's epilogue
        continue;
      }
      {
        float4* dst = reinterpret_cast<float4*>(my_slot) + (size_t)(col / 4) * kRows + trow;
#pragma unroll
        for (int i = 0; i < kColsPerWarp / 4; ++i)
          __stcg(dst + (size_t)i * kRows, make_float4(own[4 * i], own[4 * i + 1], own[4 * i + 2], own[4 * i + 3]));
      }
      // ---- partial: (M, L) beside O; counted in (and perhaps merged) after the CTA's last piece
      float* ml = reinterpret_cast<float*>(my_slot + (size_t)kRows * kD * 4);
      if (part == 0) {
        __stcg(ml + trow, M);
        __stcg(ml + kRows + trow, L);
      }
      if (!(ok = quad_sync())) break;  // s_part is rewritten by the next piece's epilogue
      if (npart < 2) partials[npart++] = pc;
    }
    // ---- publish this CTA's partial pieces (its first and / or last): every softmax thread's slot
    // writes precede the barrier (CTA-scope release / acquire); one thread counts each piece in
    // with a device-scope acquire-release atomic, and the piece that completes its item merges it
    if (ok && npart > 0) ok = soft_sync();
    if (ok && npart > 0 && tid == 0) {
      for (int i = 0; i < npart; ++i) {
        unsigned pieces = 0, cnt = 0;  // kTail: the non-empty parts of tail item q count at q
        if (stream_k) {
          const long long u0 = plan.start_of(partials[i].item);
          const int c_lo = plan.cta_of(u0), c_hi = plan.cta_of(u0 + partials[i].n_item - 1);
          for (int cx = c_lo; cx <= c_hi; ++cx) pieces += plan.seg(cx) < plan.seg(cx + 1);  // non-empty segments
          cnt = partials[i].item;
        } else {
          cnt = (-1 - partials[i].item) - tF * tS;
          pieces = (unsigned)min(partials[i].n_item, nparts((int)cnt));
        }
        s_merge[i] = atom_add_acq_rel_gpu(&counters[cnt], 1u) + 1 == pieces;
      }
    }
    if (ok && npart > 0) ok = soft_sync();
    for (int i = 0; ok && i < npart; ++i) {
      if (!s_merge[i]) continue;
      const Piece& pm = partials[i];
      const Item it = item_coords(pm);
      const int row = it.tile * kRows + trow;
      // the item's pieces: stream-K, one per CTA with a non-empty segment in [c_lo, c_hi]; kTail,
      // the non-empty parts p of tail item q, on ranks first(q) + p (slot 2 * rank + 1 each)
      int c_lo = 0, c_hi = 0, q = 0;
      if (stream_k) {
        const long long u0 = plan.start_of(pm.item);
        c_lo = plan.cta_of(u0);
        c_hi = plan.cta_of(u0 + pm.n_item - 1);
      } else {
        q = (-1 - pm.item) - tF * tS;
        c_hi = nparts(q) - 1;
      }
      auto slot_at = [&](int cx) -> const unsigned char* {  // null: no piece there
        if (!stream_k) {
          const int n = pm.n_item, w = c_hi + 1;
          if (cx * n / w == (cx + 1) * n / w) return nullptr;
          return slots + (size_t)(2 * (part_first(q) + cx) + 1) * kSlotBytes;
        }
        if (plan.seg(cx) == plan.seg(cx + 1)) return nullptr;
        return slots + (size_t)plan.slot_of(pm.item, cx) * kSlotBytes;
      };
      // the pieces' O, three slots at a time, bulk-copied into the (now idle) Q/K/V tile buffers: one
      // round trip per batch instead of one per slot; the first batch goes out before the maxima
      constexpr int kBatch = kTilesBytes / (kRows * kD * 4);
      auto issue_batch = [&](int base) {
        if (tid != 0) return;
        const unsigned char* src[kBatch];
        uint32_t bytes = 0;
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          src[u] = base + u <= c_hi ? slot_at(base + u) : nullptr;
          bytes += src[u] ? kRows * kD * 4 : 0;
        }
        // order this thread's acquired view of the partials and the previous batch's reads of the
        // buffers (generic proxy) before the bulk copies (async proxy)
        asm volatile("fence.proxy.async;" ::: "memory");
        mbar_expect_tx(bulk_bar, bytes);
#pragma unroll
        for (int u = 0; u < kBatch; ++u)
          if (src[u]) bulk_load(smem + (size_t)u * kRows * kD * 4, src[u], kRows * kD * 4, bulk_bar);
      };
      issue_batch(c_lo);
      // maxima and sums of the first 8 slots, kept for the weights; further slots (stream-K only)
      // 8 maxima at a time, their sums read again with their batch
      float m8[8], l8[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const unsigned char* sl = c_lo + u <= c_hi ? slot_at(c_lo + u) : nullptr;
        const float* mlx = sl ? reinterpret_cast<const float*>(sl + (size_t)kRows * kD * 4) : nullptr;
        m8[u] = mlx ? __ldcg(mlx + trow) : -INFINITY;
        l8[u] = mlx ? __ldcg(mlx + kRows + trow) : 0.f;
      }
      float Mx = -INFINITY;
#pragma unroll
      for (int u = 0; u < 8; ++u) Mx = fmaxf(Mx, m8[u]);
      for (int base = c_lo + 8; base <= c_hi; base += 8) {
        float mv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const unsigned char* sl = base + u <= c_hi ? slot_at(base + u) : nullptr;
          mv[u] = sl ? __ldcg(reinterpret_cast<const float*>(sl + (size_t)kRows * kD * 4) + trow) : -INFINITY;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) Mx = fmaxf(Mx, mv[u]);
      }
      float acc[kColsPerWarp], den = 0.f;
#pragma unroll
      for (int j = 0; j < kColsPerWarp; ++j) acc[j] = 0.f;
      for (int base = c_lo; ok && base <= c_hi; base += kBatch) {
        const unsigned char* sl[kBatch];
        float mk[kBatch], lk[kBatch];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          sl[u] = base + u <= c_hi ? slot_at(base + u) : nullptr;
          const int rel = base - c_lo + u;
          if (rel < 8) {  // from the registers above (a select chain: the index is not a constant)
            mk[u] = m8[0];
            lk[u] = l8[0];
#pragma unroll
            for (int k = 1; k < 8; ++k) {
              mk[u] = rel == k ? m8[k] : mk[u];
              lk[u] = rel == k ? l8[k] : lk[u];
            }
            if (!sl[u]) mk[u] = -INFINITY, lk[u] = 0.f;
          } else {
            const float* mlx = sl[u] ? reinterpret_cast<const float*>(sl[u] + (size_t)kRows * kD * 4) : nullptr;
            mk[u] = mlx ? __ldcg(mlx + trow) : -INFINITY;
            lk[u] = mlx ? __ldcg(mlx + kRows + trow) : 0.f;
          }
        }
        ok = __all_sync(0xffffffffu, wait(bulk_bar, (bulk_phase++) & 1));
        if (!ok) break;
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          if (!sl[u]) continue;
          const float wk = mk[u] == -INFINITY ? 0.f : ex2(mk[u] - Mx);
          den += wk * lk[u];
          const float4* src = reinterpret_cast<const float4*>(smem + (size_t)u * kRows * kD * 4) + (col / 4) * kRows + trow;
#pragma unroll
          for (int j = 0; j < kColsPerWarp / 4; ++j) {
            const float4 x = src[j * kRows];
            acc[4 * j] = fmaf(x.x, wk, acc[4 * j]);
            acc[4 * j + 1] = fmaf(x.y, wk, acc[4 * j + 1]);
            acc[4 * j + 2] = fmaf(x.z, wk, acc[4 * j + 2]);
            acc[4 * j + 3] = fmaf(x.w, wk, acc[4 * j + 3]);
          }
        }
        ok = soft_sync();  // the batch is read: the next may overwrite the buffers
        if (ok && base + kBatch <= c_hi) issue_batch(base + kBatch);
      }
      if (!ok) break;
      if (row < R) {
        const float inv = den > 0.f ? 1.f / den : 0.f;
        T* orow = out + ((long long)row * Hq + it.head) * kD + col;
#pragma unroll
        for (int j = 0; j < kColsPerWarp; j += 8) {
          uint4 w = make_uint4(pack2<T>(acc[j] * inv, acc[j + 1] * inv), pack2<T>(acc[j + 2] * inv, acc[j + 3] * inv),
                               pack2<T>(acc[j + 4] * inv, acc[j + 5] * inv), pack2<T>(acc[j + 6] * inv, acc[j + 7] * inv));
          *reinterpret_cast<uint4*>(orow + j) = w;
        }
      }
      if (tid == 0) counters[stream_k ? pm.item : q] = 0u;  // every piece has counted in: ready for the next call
    }
  }
  tc_fence_before();
  __syncthreads();
  if (*s_abort && tid == 0) {
    if (err) atomicOr(err, 4u);
    // let copies and MMAs already issued land before the CTA's resources go away: each barrier
    // an async unit arrives on gets a short bounded wait on both parities
    for (int b = 0; b < 2; ++b)
      for (int i = 0; i < kNumBars; ++i)
        if (i < 10 || (i >= 13 && i < 19) || i == 24) mbar_wait(bars + i, b, kAbortWaitNs);
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
  }
}

int sm_count() {
  static int cache[128] = {0};
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= 128) return 148;
  if (!cache[d]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d) != cudaSuccess || n <= 0) n = 148;
    cache[d] = n;
  }
  return cache[d];
}

template <typename T>
int launch_tc(const void* q, const void* K, const void* V, long long c_sh, long long T_cache, const int64_t* pos,
              int R, int Hq, int Hkv, float sm_scale, void* out, unsigned* err, void* ws, size_t ws_bytes,
              int force, cudaStream_t st) {
  const CUtensorMapDataType dt =
      std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap mq, mk, mv;
  if (!make_map(&mq, q, dt, kD, Hq, R, kD, (uint64_t)Hq * kD, 1, kRows) ||
      !make_map(&mk, K, dt, kD, T_cache, Hkv, kD, c_sh, kKeys, 1) ||
      !make_map(&mv, V, dt, kD, T_cache, Hkv, kD, c_sh, kKeys, 1)) {
    set_error("attn_rows: cuTensorMapEncodeTiled failed");
    return TREAD_ERR_CUDA;
  }
  static std::once_flag attr_once;
  static cudaError_t attr_rc = cudaSuccess;
  std::call_once(attr_once, [] {
    attr_rc = cudaFuncSetAttribute(attn_rows_tc_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   kSmem);
    if (attr_rc == cudaSuccess)
      attr_rc = cudaFuncSetAttribute(attn_rows_tc_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  });
  TREAD_CHECK_CUDA(attr_rc);
  const long long ntiles = ((long long)R + kRows - 1) / kRows;
  const long long nitems = (long long)Hq * ntiles;
  const int sms = sm_count();
  // Schedule (measured on B200): with a workspace, persistent CTAs (one per SM) over whole tiles,
  // longest first, the tiles left after the full rounds split into key ranges (kTail). From 64
  // rows to 8000 it is as fast as one CTA per tile or faster (up to 2x for few tiles), and faster
  // than stream-K. Without a workspace, one CTA per whole tile. force (kStreamK / kTail, from the
  // caller's flags) overrides the choice.
  const bool ws_ok = ws != nullptr && ws_bytes >= kCounterBytes + (size_t)2 * sms * kSlotBytes &&
                     nitems <= kMaxItems && ntiles <= kMaxTiles && T_cache <= (1LL << 24);
  const int mode = !ws_ok ? kWhole : force ? force : kTail;
  const float log2e = 1.4426950408889634f;
  attn_rows_tc_kernel<T><<<mode == kWhole ? (int)nitems : sms, kThreadsTC, kSmem, st>>>(
      mq, mk, mv, pos, R, Hq, Hq / Hkv, T_cache, sm_scale * log2e, static_cast<T*>(out), err,
      static_cast<unsigned char*>(mode == kWhole ? nullptr : ws), mode);
  TREAD_CHECK_LAUNCH("attn_rows_tc_kernel");
  return TREAD_OK;
}

}  // namespace

size_t attn_tc_workspace_bytes() { return kCounterBytes + (size_t)2 * sm_count() * kSlotBytes; }

// Tensor-core path for bf16/fp16 with head_dim 128; everything else runs on CUDA cores.
int attn_rows_dispatch(const void* q, const void* K, const void* V, long long c_sh, long long T_cache,
                       const int64_t* pos, int R, int Hq, int Hkv, int D, float sm_scale, void* out, int dtype,
                       unsigned* err, void* ws, size_t ws_bytes, cudaStream_t st, int flags) {
  const bool tc_ok = D == kD && (dtype == TREAD_BF16 || dtype == TREAD_F16) && !(flags & 1) &&
                     (reinterpret_cast<uintptr_t>(q) % 16 == 0) && (reinterpret_cast<uintptr_t>(K) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(V) % 16 == 0) && (c_sh * 2) % 16 == 0 && R <= 0x7fffffff - kRows &&
                     (long long)Hq * ((R + kRows - 1) / kRows) <= 0x7fffffff;
  if (!tc_ok) return attn_rows_simt(q, K, V, c_sh, T_cache, pos, R, Hq, Hkv, D, sm_scale, out, dtype, err, st);
  const int force = (flags & 2) ? kStreamK : (flags & 4) ? kTail : 0;
  if (dtype == TREAD_BF16)
    return launch_tc<__nv_bfloat16>(q, K, V, c_sh, T_cache, pos, R, Hq, Hkv, sm_scale, out, err, ws, ws_bytes, force,
                                    st);
  return launch_tc<__half>(q, K, V, c_sh, T_cache, pos, R, Hq, Hkv, sm_scale, out, err, ws, ws_bytes, force, st);
}

}  // namespace tread
