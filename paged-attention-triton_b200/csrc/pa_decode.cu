// pa_decode.cu -- paged-attention decode for B200 (sm_100a).
//
// One persistent kernel per decode step. Each warp is an independent worker:
// it owns a contiguous range of TILE-token tiles of the flattened
// (sequence, kv-head, tile) space, streams the K/V page rows of those tiles
// into shared memory with TMA (cp.async.bulk.tensor, 128-byte swizzle, an
// NS-deep mbarrier ring per warp), and runs the FP32 online softmax with both
// products on the tensor cores (mma.sync m16n8k16, K and V fed by ldmatrix).
// A worker whose range covers a whole (sequence, kv-head) writes the final
// output; otherwise it stores a partial (normalised O, LSE) and the last
// arriving worker of that segment merges the partials with the reference's
// LSE rule. No spin-waits on other CTAs: the arrival counter only decides who
// merges.
//
// Reference algorithm (paths inside bw-won/paged-attention-triton):
//   token -> page translation   paged_attention/split_kv_kernel.py:52-58
//   masked scores, online max   paged_attention/split_kv_kernel.py:68-77
//   partial O / LSE             paged_attention/split_kv_kernel.py:79-84
//   empty split, -1e30 sentinel paged_attention/split_kv_kernel.py:7-9,32-33
//   LSE reduce                  paged_attention/split_kv_kernel.py:101-122
//   split sizes                 paged_attention/torch_kernel.py:30
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <climits>
#include <mutex>

#include "pa_decode.h"
#include "fastdiv.h"

// The library can be compiled as one translation unit, or as parts in
// parallel (build.py): part 0 holds the host API and the small kernels, parts
// 1-4 instantiate the decode kernels (explicit instantiations at the end).
#if !defined(PA_PART) || PA_PART == 0
#define PA_HOST_PART 1
#else
#define PA_HOST_PART 0
#endif

namespace pa {

constexpr int kCumMax = 1024;       // rows whose tile prefix sum fits in shared memory
constexpr int kDescInts = 12;       // per-stage tile descriptor
constexpr float kSentinel = -1e30f;     // split_kv_kernel.py:8
constexpr float kValidLse = -1e29f;     // split_kv_kernel.py:9
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr unsigned long long kWaitLimitNs = 2000000000ull;   // 2 s per barrier wait
constexpr unsigned kFull = 0xffffffffu;

// Head-dimension constants (D in {64, 128, 256}).
template <int D>
struct HD {
  static constexpr int kChunks = D / 64;       // 128-byte (64-dim) chunks of one K/V row
  static constexpr int kSteps = D / 16;        // 16-dim MMA steps over a row
  static constexpr int kLaneF = D / 32;        // floats of a merge row held by one lane
  static constexpr int kSlotStride = D + 4;    // floats per shared merge row (D + LSE, 16-B aligned)
};

// Shared-memory plan of one kernel variant.
template <bool kDup, int TILE, int NW, int NS, int D>
struct Cfg {
  static constexpr int kMB = TILE / 16;            // 16-token m-blocks per tile
  // A K (or V) tile is stored box-major: for each TMA box of R token rows,
  // [chunk 0: R rows x 128 B]...[chunk D/64-1], each chunk 128-byte swizzled.
  static constexpr int kKV = TILE * D * 2;         // one K (or V) tile
  // query rows loaded with a piece's first tile (4 heads with duplicated
  // columns, else 8), rounded to the 1 KB swizzle atom
  static constexpr int kQ = ((kDup ? 4 : 8) * D * 2 + 1023) / 1024 * 1024;
  static constexpr int kStage = 2 * kKV + kQ;      // multiple of 1 KB (swizzle atom)
  static constexpr int kStagesBytes = NW * NS * kStage;
  static constexpr int kBarOff = kStagesBytes;
  static constexpr int kDescOff = kBarOff + NW * NS * 8;
  static constexpr int kCumOff = kDescOff + NW * NS * kDescInts * 4;
  // group merge area: NW arrival counters, then [NW][2][slot_cols][kSlotStride] floats
  static constexpr int kGroupOff = (kCumOff + (kCumMax + 1) * 4 + 15) & ~15;
  static constexpr int kGroupCntBytes = (NW * 4 + 15) & ~15;
  static constexpr int kSmemBase = kGroupOff + kGroupCntBytes + 1024;  // + alignment slack
  static constexpr int kGroupSlotBytes = NW * 2 * HD<D>::kSlotStride * 4;   // per slot column
};

struct KParams {
  const char* q;            // bytes
  long long q_sb, q_sh;     // bytes
  char* out;
  long long o_sb, o_sh;     // bytes
  float* lse;
  const int* bt;
  long long bt_sb;          // elements
  int max_blocks;
  const int* seq_lens;
  int seq_len;              // uniform length (seq_lens == nullptr)
  int B, Hq, Hkv, G, QC, bs, NB;
  int bs_log2;              // log2(bs) if a power of two, else -1
  int ns;                   // 0: balanced schedule
  float scale_log2;         // softmax scale * log2(e)
  float* o_part;            // split: [B, Hq, ns, D]; balanced: [2W, 8, D]
  float* lse_part;          // split: [B, Hq, ns];    balanced: [2W, 8]
  int* counters;
  unsigned* status;
  int R;                    // rows per TMA box (gcd(bs, TILE))
  int lspt;                 // log2(TILE / R): boxes per tile
  int lR;                   // log2(R)
  int W;                    // workers
  int slot_cols;            // partial slot width: min(G, 8) query heads
  int gsz;                  // warps per merge group (NW, or 1 for short segments whose
                            // merge rows do not fit in shared memory)
  int zero_rows;            // 1: some row may have length 0 (the output pre-pass runs)
  // Balanced schedule, computed on the host: the unit count and range sizes
  // (valid when every row has the same length), and the launch-invariant
  // divisors of the unit decode as multiply-shift constants.
  int U, P, Pw;             // units; units per group range; per warp range
  int nt_u, per_row;        // tiles per segment, units per row (same-length rows)
  FastDiv div_row;          // by per_row
  FastDiv div_nt;           // by nt_u
  FastDiv div_qc;           // by QC
  FastDiv div_bs;           // by bs (pages that are not a power of two)
  FastDiv div_ng;           // by the number of groups (P with per-row lengths)
  float* wslots;            // warps' merge rows in global memory (null: shared memory)
  int post_merge;           // 1: segments that cross groups merge in merge_segments_kernel
  // Per-row lengths, whole-CTA groups: group boundaries move to the nearest
  // segment boundary when segments are short (max_nt: tiles of the longest
  // possible segment), so no segment crosses a group and every merge stays in
  // shared memory.
  int snap, max_nt;
  // Same-length rows, segments longer than a CTA's share: a thread-block
  // cluster of `clu` CTAs per segment (0: off), each CTA one contiguous part of
  // it; the CTAs' pieces meet in distributed shared memory (at byte offset
  // clu_off of every CTA's aligned shared memory) instead of through L2.
  int clu, clu_off;
};
// ----------------------------------------------------------------------------
// PTX helpers
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Waits for the barrier phase with a wall-clock bound; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity,
                                          unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - t0 > limit_ns) return false;
  }
}

__device__ __forceinline__ void tma_load_5d(uint32_t dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, int c3, int c4, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ uint32_t movm_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// Distributed shared memory of a thread-block cluster.
__device__ __forceinline__ uint32_t cluster_map(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
// One thread's arrival on an mbarrier in another CTA of the cluster; its
// earlier stores to that CTA's shared memory are visible to whoever completes
// a wait on the barrier's phase with cluster-scope acquire.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t remote_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote_bar)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

template <typename T>
struct Mma;

template <>
struct Mma<__half> {
  __device__ __forceinline__ static void run(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                             uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  // Rounds p to the operand type and returns (hi, lo) with hi + lo ~= p.
  __device__ __forceinline__ static void split(float p, uint16_t& hi, uint16_t& lo) {
    const __half h = __float2half_rn(p);
    const __half l = __float2half_rn(p - __half2float(h));
    hi = __half_as_ushort(h);
    lo = __half_as_ushort(l);
  }
  __device__ __forceinline__ static uint16_t from_float(float x) {
    return __half_as_ushort(__float2half_rn(x));
  }
  // Packed (p0, p1) rounded to the operand type (hi) and the rounded residual (lo).
  __device__ __forceinline__ static void split2(float p0, float p1, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(p0, p1);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(p0 - hf.x, p1 - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
  }
};

template <>
struct Mma<__nv_bfloat16> {
  __device__ __forceinline__ static void run(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                             uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  __device__ __forceinline__ static void split(float p, uint16_t& hi, uint16_t& lo) {
    const __nv_bfloat16 h = __float2bfloat16_rn(p);
    const __nv_bfloat16 l = __float2bfloat16_rn(p - __bfloat162float(h));
    hi = __bfloat16_as_ushort(h);
    lo = __bfloat16_as_ushort(l);
  }
  __device__ __forceinline__ static uint16_t from_float(float x) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(x));
  }
  __device__ __forceinline__ static void split2(float p0, float p1, uint32_t& hi, uint32_t& lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(p0, p1);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(p0 - hf.x, p1 - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
  }
};

__device__ __forceinline__ uint32_t pack16(uint16_t lo, uint16_t hi) {
  return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

// ----------------------------------------------------------------------------

// ----------------------------------------------------------------------------
// Work decomposition
// ----------------------------------------------------------------------------
// A unit is one TILE-token tile of one segment; a segment is one row b and one
// (kv head, query chunk) pair, query chunk qc holding query heads
// kvh*G + qc*8 .. +min(8, G - qc*8).
//
// Balanced schedule: units are flattened in (b, kvh, qc, tile) order. Group g
// (the gsz warps of one CTA, or a single warp) owns [g*P, min(U, (g+1)*P)),
// and warp i of the group the contiguous part [gr0 + i*Pw, ...). A piece is the
// part of a segment inside one warp's range. Pieces of a segment inside one
// group are merged in shared memory by the warp that finishes last; the
// group's piece of a segment that crosses groups goes to a global partial slot
// (2g: the piece starts the group's range, 2g+1: it ends it), and the group
// that finishes the segment last merges those.
//
// Split schedule (the reference's): worker w owns split s of one segment; its
// single range is the split's tiles, and its partial is the split's row.

__device__ __forceinline__ int clamp_len(const KParams& p, int s, bool& bad) {
  const int cap = p.max_blocks * p.bs;
  if (s < 0) { bad = true; return 0; }
  if (s > cap) { bad = true; return cap; }
  return s;
}

// Length of row b: the uniform length, or (kCum: per-row lengths) seq_lens[b].
template <bool kCum>
__device__ __forceinline__ int row_len(const KParams& p, int b) {
  if constexpr (!kCum) return p.seq_len;
  bool bad = false;
  return clamp_len(p, __ldg(p.seq_lens + b), bad);
}

// Largest b in [0, B) with cum[b] <= u (cum non-decreasing, cum[0] = 0).
__device__ __forceinline__ int find_row(const int* cum, int B, int u) {
  int lo = 0, hi = B - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cum[mid] <= u) lo = mid; else hi = mid - 1;
  }
  return lo;
}

struct Ranges {       // balanced schedule of one warp
  int U;              // units in the step
  int P, Pw;          // units per group range, per warp range
  int g, gi;          // group, warp index inside the group
  int gr0, gr1;       // group range
  int wr0, wr1;       // warp range
};

struct Work {         // split schedule: the worker's one piece
  int b, kvh, qc, s, t0, t1, tl0, n;
};

// Position of a tile: segment, tile within it, segment length in tiles.
struct Cursor {
  int b, kvh, qc;
  int tile, nt, S;
  int seg_lo;         // unit index of the segment's tile 0 (balanced)
};

template <int TILE, bool kCum>
__device__ __forceinline__ void decode_unit(Cursor& c, const KParams& p, const int* cum, int u) {
  int row_base;
  if constexpr (kCum) {
    c.b = find_row(cum, p.B, u);
    row_base = cum[c.b];
    c.S = row_len<true>(p, c.b);
    c.nt = (c.S + TILE - 1) / TILE;
  } else {
    c.S = p.seq_len;
    c.nt = p.nt_u;
    c.b = static_cast<int>(fast_div(static_cast<uint32_t>(u), p.div_row));
    row_base = c.b * p.per_row;
  }
  const int r = u - row_base;
  const int seg = kCum ? r / c.nt : static_cast<int>(fast_div(static_cast<uint32_t>(r), p.div_nt));
  c.tile = r - seg * c.nt;
  c.kvh = p.QC == 1 ? seg : static_cast<int>(fast_div(static_cast<uint32_t>(seg), p.div_qc));
  c.qc = seg - c.kvh * p.QC;
  c.seg_lo = row_base + seg * c.nt;
}

// Next unit in flattened order (balanced).
template <int TILE, bool kCum>
__device__ __forceinline__ void cursor_next(Cursor& c, const KParams& p) {
  if (++c.tile < c.nt) return;
  c.tile = 0;
  c.seg_lo += c.nt;
  if (++c.qc < p.QC) return;
  c.qc = 0;
  if (++c.kvh < p.Hkv) return;
  c.kvh = 0;
  do {   // next row that owns tiles (rows of length 0 own none)
    if (c.b + 1 >= p.B) { c.nt = 1; return; }   // past the end: never used
    ++c.b;
    c.S = row_len<kCum>(p, c.b);
    c.nt = (c.S + TILE - 1) / TILE;
  } while (c.nt == 0);
}

// Flags of a tile's piece (balanced).
constexpr int kFirst = 1;      // first tile of the warp's piece
constexpr int kLast = 2;       // last tile of the warp's piece
constexpr int kWarpSeg = 4;    // the warp's piece is the whole segment
constexpr int kWarpGroup = 8;  // the warp's piece is the group's whole piece
constexpr int kGroupSeg = 16;  // the group's piece is the whole segment

template <int TILE>
__device__ __forceinline__ void piece_of(const Cursor& c, const Ranges& rg, int& t0, int& t1,
                                         int& flags) {
  const int u = c.seg_lo + c.tile;
  const int seg_hi = c.seg_lo + c.nt;
  const int plo = max(c.seg_lo, rg.wr0), phi = min(seg_hi, rg.wr1);
  const int glo = max(c.seg_lo, rg.gr0), ghi = min(seg_hi, rg.gr1);
  t0 = (plo - c.seg_lo) * TILE;
  t1 = min(c.S, (phi - c.seg_lo) * TILE);
  flags = (u == plo ? kFirst : 0) | (u == phi - 1 ? kLast : 0) |
          ((plo == c.seg_lo && phi == seg_hi) ? kWarpSeg : 0) |
          ((plo == glo && phi == ghi) ? kWarpGroup : 0) |
          ((glo == c.seg_lo && ghi == seg_hi) ? kGroupSeg : 0);
}

// One warp's arrival on a counter that elects the last of `n` arrivals (the
// warp that merges). Every lane's writes before the call are visible to the
// last arriver, and the last arriver's lanes see every other arriver's writes:
// a warp barrier orders the lanes' writes before lane 0's acquire-release
// atomic, a second one orders that acquire before the lanes' later reads (no
// sequentially consistent fence is needed). kGpu: a counter in global memory
// at GPU scope; else one in shared memory at CTA scope.
template <bool kGpu>
__device__ __forceinline__ bool arrive_elect_last(int* counter, int n, int lane) {
  __syncwarp();
  int old = 0;
  if (lane == 0) {
    if constexpr (kGpu)
      asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;"
                   : "=r"(old) : "l"(counter) : "memory");
    else
      asm volatile("atom.acq_rel.cta.shared::cta.add.s32 %0, [%1], 1;"
                   : "=r"(old) : "r"(smem_u32(counter)) : "memory");
  }
  const bool last = __shfl_sync(kFull, old, 0) == n - 1;
  __syncwarp();
  return last;
}

__device__ __forceinline__ void flag(const KParams& p, unsigned bits) {
  if (p.status) atomicOr(p.status, bits);
}

// Block-table page and slot of this lane's TMA box in a batch of tiles: lane L
// serves box (L & (spt-1)) of tile (L >> lspt) of the batch [u0, u1) (units of
// the warp range, or tile ordinals of a split). INT_MIN: the box holds no token
// of its piece (not loaded; the consumer masks it). One load per lane.
template <int TILE, bool kSplit, bool kCum>
__device__ __forceinline__ void batch_pages(const KParams& p, const int* cum, const Ranges& rg,
                                            const Work& w, int u0, int u1, int lane, int& phys,
                                            int& slot) {
  const int ord = lane >> p.lspt;
  const int j = lane & ((1 << p.lspt) - 1);
  long long off = -1;
  slot = 0;
  if (u0 + ord < u1) {
    int tile, b, t0, t1;
    if constexpr (!kSplit) {
      Cursor c;
      decode_unit<TILE, kCum>(c, p, cum, u0 + ord);
      int fl;
      piece_of<TILE>(c, rg, t0, t1, fl);
      tile = c.tile;
      b = c.b;
    } else {
      tile = w.tl0 + u0 + ord;
      b = w.b;
      t0 = w.t0;
      t1 = w.t1;
    }
    const int tt = tile * TILE + j * p.R;
    if (tt < t1 && tt + p.R > t0) {
      const int lp = p.bs_log2 >= 0 ? (tt >> p.bs_log2)
                                    : static_cast<int>(fast_div(static_cast<uint32_t>(tt), p.div_bs));
      off = static_cast<long long>(b) * p.bt_sb + lp;
      slot = tt - lp * p.bs;
    }
  }
  phys = off >= 0 ? __ldg(p.bt + off) : INT_MIN;
}

// ----------------------------------------------------------------------------
// Merging pieces
// ----------------------------------------------------------------------------
// One lane's share of a merge row: floats [lane * N, lane * N + N).
template <int N>
struct RowV {
  float f[N];
};

template <bool kGlobal, int N>
__device__ __forceinline__ RowV<N> load_row(const float* row, int lane) {
  RowV<N> r;
  const float* q = row + lane * N;
  if constexpr (N == 2) {
    const float2* q2 = reinterpret_cast<const float2*>(q);
    const float2 t = kGlobal ? __ldcg(q2) : *q2;
    r.f[0] = t.x;
    r.f[1] = t.y;
  } else {
#pragma unroll
    for (int i = 0; i < N; i += 4) {
      const float4* q4 = reinterpret_cast<const float4*>(q + i);
      const float4 t = kGlobal ? __ldcg(q4) : *q4;
      r.f[i] = t.x;
      r.f[i + 1] = t.y;
      r.f[i + 2] = t.z;
      r.f[i + 3] = t.w;
    }
  }
  return r;
}

template <int N>
__device__ __forceinline__ void store_row(float* row, int lane, const RowV<N>& r) {
  float* q = row + lane * N;
  if constexpr (N == 2) {
    *reinterpret_cast<float2*>(q) = make_float2(r.f[0], r.f[1]);
  } else {
#pragma unroll
    for (int i = 0; i < N; i += 4)
      *reinterpret_cast<float4*>(q + i) = make_float4(r.f[i], r.f[i + 1], r.f[i + 2], r.f[i + 3]);
  }
}

// split_kv_kernel.py:101-122: skip lse <= -1e29, merge by running max, divide
// by max(sum, 1e-20); no valid piece gives 0 and LSE -1e30. `src(k, row, lse)`
// locates piece k's normalised row (D floats) and LSE; rows are read from
// global memory through L2 (kGlobal) or from shared memory. Each lane returns
// its D/32 dims.
template <bool kGlobal, int D, class Src>
__device__ __forceinline__ void merge_rows(int n, int lane, const Src& src,
                                           RowV<HD<D>::kLaneF>& out, float& lse_out) {
  constexpr int N = HD<D>::kLaneF;
  constexpr int kBatch = 8;   // rows in flight per lane
  auto ld_lse = [&](int k) {
    const float* row;
    const float* lp;
    src(k, row, lp);
    return kGlobal ? __ldcg(lp) : *lp;
  };
  auto ld_row = [&](int k) {
    const float* row;
    const float* lp;
    src(k, row, lp);
    return load_row<kGlobal, N>(row, lane);
  };
  RowV<N> zero;
#pragma unroll
  for (int i = 0; i < N; ++i) zero.f[i] = 0.f;
  RowV<N> v[kBatch];
  RowV<N> a = zero;
  if (n <= kBatch) {
    // At most one batch (the shared-memory merges and most group merges): one
    // straight pass, every lane reading all LSEs (a broadcast) and its share
    // of every row; no loops or shuffles on the tail of the step.
    float l[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      l[u] = (u < n) ? ld_lse(u) : kSentinel;
      v[u] = (u < n) ? ld_row(u) : zero;
    }
    float gmax = kValidLse;
#pragma unroll
    for (int u = 0; u < kBatch; ++u)
      if (l[u] > kValidLse) gmax = fmaxf(gmax, l[u]);
    float gsum = 0.f;
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const float wgt = (l[u] > kValidLse) ? exp2f((l[u] - gmax) * kLog2e) : 0.f;
      gsum += wgt;
#pragma unroll
      for (int i = 0; i < N; ++i) a.f[i] = fmaf(wgt, v[u].f[i], a.f[i]);
    }
    const float inv = __fdividef(1.f, fmaxf(gsum, 1e-20f));
#pragma unroll
    for (int i = 0; i < N; ++i) out.f[i] = a.f[i] * inv;
    lse_out = gsum > 0.f ? gmax + __logf(gsum) : kSentinel;
    return;
  }
  const float l0 = (lane < n) ? ld_lse(lane) : kValidLse;
#pragma unroll
  for (int u = 0; u < kBatch; ++u) v[u] = (u < n) ? ld_row(u) : zero;
  float gmax = (l0 > kValidLse) ? l0 : kValidLse;
  for (int k = lane + 32; k < n; k += 32) {
    const float l = ld_lse(k);
    if (l > kValidLse) gmax = fmaxf(gmax, l);
  }
#pragma unroll
  for (int o2 = 16; o2 > 0; o2 >>= 1) gmax = fmaxf(gmax, __shfl_xor_sync(kFull, gmax, o2));
  float gsum = 0.f;
  for (int base = 0; base < n; base += 32) {
    const float lb = (base == 0) ? l0 : ((base + lane < n) ? ld_lse(base + lane) : kValidLse);
    const float wl = (lb > kValidLse) ? exp2f((lb - gmax) * kLog2e) : 0.f;
    float ws = wl;
#pragma unroll
    for (int o2 = 16; o2 > 0; o2 >>= 1) ws += __shfl_xor_sync(kFull, ws, o2);
    gsum += ws;
    const int cnt = min(32, n - base);
    for (int k0 = 0; k0 < cnt; k0 += kBatch) {
      if (base + k0 > 0) {
#pragma unroll
        for (int u = 0; u < kBatch; ++u)
          v[u] = (k0 + u < cnt) ? ld_row(base + k0 + u) : zero;
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const float wgt = __shfl_sync(kFull, wl, (k0 + u) & 31);
        if (k0 + u < cnt && wgt > 0.f) {
#pragma unroll
          for (int i = 0; i < N; ++i) a.f[i] = fmaf(wgt, v[u].f[i], a.f[i]);
        }
      }
    }
  }
  const float inv = 1.f / fmaxf(gsum, 1e-20f);
#pragma unroll
  for (int i = 0; i < N; ++i) out.f[i] = a.f[i] * inv;
  lse_out = gsum > 0.f ? gmax + logf(gsum) : kSentinel;
}

// The same rule over rows in shared memory, as one compact loop with a running
// max (the order of split_kv_kernel.py:105-118): the merge runs once per
// piece on the step's tail, where straight-line code is paid for in
// instruction fetch, and shared-memory loads are short enough not to need
// batching.
template <int D, class Src>
__device__ __forceinline__ void merge_rows_smem(int n, int lane, const Src& src,
                                                RowV<HD<D>::kLaneF>& out, float& lse_out) {
  constexpr int N = HD<D>::kLaneF;
  float m = kValidLse, sum = 0.f;
  RowV<N> a;
#pragma unroll
  for (int i = 0; i < N; ++i) a.f[i] = 0.f;
#pragma unroll 1
  for (int k = 0; k < n; ++k) {
    const float* row;
    const float* lp;
    src(k, row, lp);
    const float l = *lp;
    if (l > kValidLse) {
      const RowV<N> v = load_row<false, N>(row, lane);
      const float mn = fmaxf(m, l);
      const float f = exp2f((m - mn) * kLog2e);
      const float wgt = exp2f((l - mn) * kLog2e);
      sum = fmaf(sum, f, wgt);
#pragma unroll
      for (int i = 0; i < N; ++i) a.f[i] = fmaf(a.f[i], f, wgt * v.f[i]);
      m = mn;
    }
  }
  const float inv = __fdividef(1.f, fmaxf(sum, 1e-20f));
#pragma unroll
  for (int i = 0; i < N; ++i) out.f[i] = a.f[i] * inv;
  lse_out = sum > 0.f ? m + __logf(sum) : kSentinel;
}

// Final output row of (b, hq): this lane's D/32 dims in the output dtype.
template <typename T, int D>
__device__ __forceinline__ void store_out(const KParams& p, int b, int hq, int lane,
                                          const RowV<HD<D>::kLaneF>& o, float lse) {
  constexpr int N = HD<D>::kLaneF;
  char* dst = p.out + b * p.o_sb + hq * p.o_sh + lane * N * 2;
  uint32_t w[N / 2];
#pragma unroll
  for (int i = 0; i < N / 2; ++i)
    w[i] = pack16(Mma<T>::from_float(o.f[2 * i]), Mma<T>::from_float(o.f[2 * i + 1]));
  if constexpr (N == 2) {
    *reinterpret_cast<uint32_t*>(dst) = w[0];
  } else if constexpr (N == 4) {
    *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
  } else {
    *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  if (lane == 0 && p.lse) p.lse[b * p.Hq + hq] = lse;
}

// Global partial slot of group g's piece: row of column j.
template <int D>
__device__ __forceinline__ float* gslot_row(const KParams& p, long long slot, int j) {
  return p.o_part + (slot * p.slot_cols + j) * D;
}
__device__ __forceinline__ float* gslot_lse(const KParams& p, long long slot, int j) {
  return p.lse_part + slot * p.slot_cols + j;
}

// The last group to finish a segment merges the groups' partials.
template <typename T, int D>
__device__ __forceinline__ void merge_groups(const KParams& p, const Ranges& rg, int b, int kvh,
                                             int qc, int gc, int seg_lo, int seg_hi, int lane) {
  const int g_first = seg_lo / rg.P;
  const int n = (seg_hi - 1) / rg.P - g_first + 1;
  auto slot_of = [&](int k) {
    const int g = g_first + k;
    return 2ll * g + (max(seg_lo, g * rg.P) == g * rg.P ? 0 : 1);
  };
  if (n <= 4) {
    // Few pieces (short segments split between neighbouring groups): the
    // pieces of up to 4 query columns are loaded in one L2 round trip instead
    // of one per column (each one is ~1 us while the grid saturates DRAM).
    constexpr int N = HD<D>::kLaneF;
    const float* rows[4];   // piece k's row of column 0, and its LSE
    const float* lses[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const long long sl = slot_of(min(k, n - 1));
      rows[k] = gslot_row<D>(p, sl, 0) + lane * N;
      lses[k] = gslot_lse(p, sl, 0);
    }
    for (int j0 = 0; j0 < gc; j0 += 4) {
      float l[4][4];
      RowV<N> v[4][4];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (j0 + jj < gc && k < n) {
            l[jj][k] = __ldcg(lses[k] + j0 + jj);
            v[jj][k] = load_row<true, N>(rows[k] + (j0 + jj) * D, 0);
          } else {
            l[jj][k] = kSentinel;
#pragma unroll
            for (int i = 0; i < N; ++i) v[jj][k].f[i] = 0.f;
          }
        }
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        if (j0 + jj >= gc) break;
        // split_kv_kernel.py:101-122
        float gmax = kValidLse;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (l[jj][k] > kValidLse) gmax = fmaxf(gmax, l[jj][k]);
        float gsum = 0.f;
        RowV<N> a;
#pragma unroll
        for (int i = 0; i < N; ++i) a.f[i] = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float wgt = (l[jj][k] > kValidLse) ? exp2f((l[jj][k] - gmax) * kLog2e) : 0.f;
          gsum += wgt;
#pragma unroll
          for (int i = 0; i < N; ++i) a.f[i] = fmaf(wgt, v[jj][k].f[i], a.f[i]);
        }
        const float inv = __fdividef(1.f, fmaxf(gsum, 1e-20f));
#pragma unroll
        for (int i = 0; i < N; ++i) a.f[i] *= inv;
        store_out<T, D>(p, b, kvh * p.G + qc * 8 + j0 + jj, lane, a,
                        gsum > 0.f ? gmax + __logf(gsum) : kSentinel);
      }
    }
    return;
  }
  for (int j = 0; j < gc; ++j) {
    auto src = [&](int k, const float*& row, const float*& lp) {
      const int g = g_first + k;
      const long long sl = 2ll * g + (max(seg_lo, g * rg.P) == g * rg.P ? 0 : 1);
      row = gslot_row<D>(p, sl, j);
      lp = gslot_lse(p, sl, j);
    };
    RowV<HD<D>::kLaneF> o;
    float lse;
    merge_rows<true, D>(n, lane, src, o, lse);
    store_out<T, D>(p, b, kvh * p.G + qc * 8 + j, lane, o, lse);
  }
}

// Split schedule: the last split of a segment merges rows [b, hq, 0..ns).
template <typename T, int D>
__device__ __forceinline__ void merge_splits(const KParams& p, int b, int kvh, int qc, int gc,
                                             int lane) {
  for (int j = 0; j < gc; ++j) {
    const int hq = kvh * p.G + qc * 8 + j;
    const long long row0 = (static_cast<long long>(b) * p.Hq + hq) * p.ns;
    auto src = [&](int k, const float*& row, const float*& lp) {
      row = p.o_part + (row0 + k) * D;
      lp = p.lse_part + row0 + k;
    };
    RowV<HD<D>::kLaneF> o;
    float lse;
    merge_rows<true, D>(p.ns, lane, src, o, lse);
    store_out<T, D>(p, b, hq, lane, o, lse);
  }
}


// Cluster mode, rank 0 of the cluster: once every CTA of the cluster has
// pushed its piece of the segment (`seg`, in (row, KV head, query chunk)
// order) into this CTA's shared memory (`crow`: [clu][slot_cols][D + 4]
// floats, the LSE at D) and arrived on `cbar`, merge the pieces with the
// reference's rule (split_kv_kernel.py:101-122) and write O and LSE. The wait
// is bounded (four times a copy wait, as a pushing CTA may itself have waited
// out one): on timeout the status word gets PA_STATUS_TIMEOUT and nothing is
// written.
template <typename T, int D, int NW>
__device__ __forceinline__ void merge_cluster(const KParams& p, const float* crow, uint32_t cbar,
                                              int seg, int warp, int lane) {
  constexpr int N = HD<D>::kLaneF;
  const int per_b = p.Hkv * p.QC;
  const int b = seg / per_b;
  const int kvh = (seg - b * per_b) / p.QC;
  const int qc = seg - b * per_b - kvh * p.QC;
  const int gc = min(8, p.G - qc * 8);
  if (warp >= gc) return;
  if (!mbar_try_wait_cluster(cbar, 0)) {
    const unsigned long long t0 = global_ns();
    while (!mbar_try_wait_cluster(cbar, 0)) {
      if (global_ns() - t0 > 4 * kWaitLimitNs) {
        if (lane == 0 && p.status) atomicOr(p.status, PA_STATUS_TIMEOUT);
        return;
      }
    }
  }
  for (int j = warp; j < gc; j += NW) {
    // One compact loop with a running max (the order of split_kv_kernel.py:105-118):
    // this code runs once per step, on its critical path, where unrolled code is
    // paid for in instruction fetch.
    float m = kValidLse, sum = 0.f;
    RowV<N> a;
#pragma unroll
    for (int i = 0; i < N; ++i) a.f[i] = 0.f;
#pragma unroll 1
    for (int k = 0; k < p.clu; ++k) {
      const float* row = crow + (k * p.slot_cols + j) * HD<D>::kSlotStride;
      const float l = row[D];
      if (l > kValidLse) {
        const RowV<N> v = load_row<false, N>(row, lane);
        const float mn = fmaxf(m, l);
        const float f = exp2f((m - mn) * kLog2e);
        const float wgt = exp2f((l - mn) * kLog2e);
        sum = fmaf(sum, f, wgt);
#pragma unroll
        for (int i = 0; i < N; ++i) a.f[i] = fmaf(a.f[i], f, wgt * v.f[i]);
        m = mn;
      }
    }
    const float inv = __fdividef(1.f, fmaxf(sum, 1e-20f));
#pragma unroll
    for (int i = 0; i < N; ++i) a.f[i] *= inv;
    store_out<T, D>(p, b, kvh * p.G + qc * 8 + j, lane, a, sum > 0.f ? m + __logf(sum) : kSentinel);
  }
}

// Cold paths, out of line so that the hot path's straight-line code does not
// interleave with them (the short steps are bound by instruction fetch).

// A barrier wait gave up: flag it and wait (bounded) for the `more` copies
// still in flight on the other stages, so that none lands after the exit.
template <int NS>
__device__ __noinline__ void drain_after_timeout(unsigned* status, uint32_t bar0, int st,
                                                 uint32_t phase, int more,
                                                 unsigned long long limit_ns = kWaitLimitNs) {
  if (status) atomicOr(status, PA_STATUS_TIMEOUT);
  for (int k = 1; k < NS && k <= more; ++k) {
    const int s2 = (st + k) % NS;
    mbar_wait(bar0 + s2 * 8, (phase >> s2) & 1, limit_ns);
  }
}

// Rows of length 0 own no tile: O = 0 and LSE = -1e30 (split_kv_kernel.py:101,120).
// With per-row lengths a row is empty when its tile prefix sum does not grow
// (negative lengths count as 0 and are flagged by the prefix-sum pass).
template <int D, bool kCum>
__device__ __noinline__ void zero_length_rows(int B, int Hq, char* out, long long o_sb,
                                              long long o_sh, float* lse, const int* cum,
                                              int seq_len) {
  for (int b = blockIdx.x; b < B; b += gridDim.x) {
    const bool empty = kCum ? (cum[b + 1] == cum[b]) : (seq_len == 0);
    if (!empty) continue;
    for (int idx = threadIdx.x; idx < Hq * (D / 8); idx += blockDim.x) {
      const int h = idx / (D / 8), c = idx % (D / 8);
      *reinterpret_cast<uint4*>(out + b * o_sb + h * o_sh + c * 16) = make_uint4(0, 0, 0, 0);
    }
    if (lse)
      for (int h = threadIdx.x; h < Hq; h += blockDim.x) lse[b * Hq + h] = kSentinel;
  }
}

// ----------------------------------------------------------------------------
// Kernel
// ----------------------------------------------------------------------------
template <typename T, bool kDup, int TILE, int NW, int NS, int D, bool kSplit, bool kCum,
          bool kClu>
__global__ void __launch_bounds__(NW * 32, 1)
    pa_decode_kernel(const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const KParams p) {
  using C = Cfg<kDup, TILE, NW, NS, D>;
  using H = HD<D>;
  constexpr int kMB = C::kMB;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  int* descs = reinterpret_cast<int*>(smem + C::kDescOff);
  int* cum = reinterpret_cast<int*>(smem + C::kCumOff);
  int* gcnt = reinterpret_cast<int*>(smem + C::kGroupOff);         // [NW] arrival counters
  // The warps' merge rows ([NW][2][slot_cols][D + 4] floats per CTA): shared
  // memory when they fit beside the stages, else this CTA's part of the
  // workspace (same-CTA writers and reader, ordered by the CTA-scope fences).
  float* gslots = p.wslots ? p.wslots + static_cast<size_t>(blockIdx.x) * NW * 2 * p.slot_cols *
                                            H::kSlotStride
                           : reinterpret_cast<float*>(smem + C::kGroupOff + C::kGroupCntBytes);
  // Cluster mode: rank 0's arrival barrier for the CTAs' pieces (cbar), then
  // the pieces themselves ([clu][slot_cols][D + 4] floats; every CTA carves
  // the same layout, only rank 0's is used). crank / cid: this CTA's rank in
  // its cluster and the cluster's index, which is its segment.
  float* cslot = kClu ? reinterpret_cast<float*>(smem + p.clu_off + 16) : nullptr;
  const uint32_t cbar = kClu ? smem_u32(smem + p.clu_off) : 0u;
  uint32_t crank = 0, cid = 0;
  if constexpr (kClu) {
    asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(crank));
    asm("mov.u32 %0, %%clusterid.x;" : "=r"(cid));
  }
  __shared__ int warp_tot[NW];
  // Cross-group publishes waiting until the warp has issued all its copies:
  // [warp][2 entries][b, kvh, qc, gc, seg_lo, seg_hi].
  __shared__ int pend_rec[kSplit ? 1 : NW][2][6];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmK)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmV)) : "memory");
  }
  if (lane == 0) {
    for (int s = 0; s < NS; ++s) mbar_init(smem_u32(&bars[warp * NS + s]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (threadIdx.x < NW) gcnt[threadIdx.x] = 0;
  // The warp's own barriers are initialised before any of its lanes issues a
  // copy; the CTA-wide barrier that publishes gcnt comes after the first
  // copies are in flight.
  __syncwarp();
  if constexpr (kClu) {
    // One arrival per lane of each CTA's pushing warp. The cluster barrier's
    // arrive here and wait after the first copies make the initialisation
    // visible to every CTA before any of them can push.
    if (threadIdx.x == 0) {
      mbar_init(cbar, static_cast<uint32_t>(p.clu) * 32u);
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  }

  // ---------------------------------------------------------------- schedule
  const int wid = blockIdx.x * NW + warp;
  Ranges rg;
  rg.U = rg.P = rg.Pw = rg.g = rg.gi = rg.gr0 = rg.gr1 = rg.wr0 = rg.wr1 = 0;
  auto set_ranges = [&](int U, int P, int Pw) {
    rg.U = U;
    rg.P = P;
    rg.Pw = Pw;
    // groups are whole CTAs (gsz == NW) or single warps (gsz == 1)
    rg.g = p.gsz == 1 ? wid : static_cast<int>(blockIdx.x);
    rg.gi = p.gsz == 1 ? 0 : warp;
    rg.gr0 = min(rg.U, rg.g * rg.P);
    rg.gr1 = min(rg.U, rg.gr0 + rg.P);
    rg.wr0 = min(rg.gr1, rg.gr0 + rg.gi * rg.Pw);
    rg.wr1 = min(rg.gr1, rg.wr0 + rg.Pw);
  };
  // Same-length rows: the ranges need no memory, so they are set before the wait.
  if (!kSplit && !kCum) {
    set_ranges(p.U, p.P, p.Pw);
    if constexpr (kClu) {
      // cluster c owns segment c; its CTA of rank r the units
      // [r * P, (r + 1) * P) of that segment (the host sizes P so that every
      // rank has some)
      const int s0 = static_cast<int>(cid) * p.nt_u;
      rg.gr0 = s0 + static_cast<int>(crank) * p.P;
      rg.gr1 = min(rg.gr0 + p.P, s0 + p.nt_u);
      rg.wr0 = min(rg.gr1, rg.gr0 + rg.gi * rg.Pw);
      rg.wr1 = min(rg.gr1, rg.wr0 + rg.Pw);
    }
  }

  // Programmatic dependent launch: everything above touches no global memory;
  // from here on the kernel reads inputs (and writes outputs, partials and
  // counters) that the previous kernel in the stream may still be using.
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // Balanced schedule with per-row lengths: per-row tile prefix sums.
  if (!kSplit && kCum) {
    const int B = p.B;
    const int nseg = p.Hkv * p.QC;
    const int chunk = (B + blockDim.x - 1) / blockDim.x;
    const int lo = min(B, static_cast<int>(threadIdx.x) * chunk);
    const int hi = min(B, lo + chunk);
    bool bad = false;
    int local = 0;
    for (int b = lo; b < hi; ++b) {
      const int S = clamp_len(p, __ldg(p.seq_lens + b), bad);
      local += nseg * ((S + TILE - 1) / TILE);
    }
    if (bad && blockIdx.x == 0) flag(p, PA_STATUS_BAD_SEQLEN);
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    int before = 0;
    for (int k = 0; k < warp; ++k) before += warp_tot[k];
    int run = before + incl - local;
    for (int b = lo; b < hi; ++b) {
      cum[b] = run;
      const int S = clamp_len(p, __ldg(p.seq_lens + b), bad);
      run += nseg * ((S + TILE - 1) / TILE);
    }
    if (threadIdx.x == blockDim.x - 1) cum[B] = before + incl;
    __syncthreads();
  }

  const int G = p.G;
  const int spt_mask = (1 << p.lspt) - 1;
  const int bt_tiles = 32 >> p.lspt;          // tiles per page batch (one box per lane)
  Work w;
  w.b = w.kvh = w.qc = w.s = w.t0 = w.t1 = w.tl0 = w.n = 0;
  int n_tiles = 0;
  if (!kSplit) {
    if (kCum) {
      const int U = cum[p.B];
      const int P = max(static_cast<int>(fast_div(static_cast<uint32_t>(U) + p.div_ng.d - 1,
                                                  p.div_ng)),
                        p.gsz);
      set_ranges(U, P, p.gsz == 1 ? P : (P + NW - 1) / NW);
      if (p.snap && P >= 8 * p.max_nt) {
        // Both CTAs that share a boundary compute the same snapped value; a
        // boundary moves by at most half a segment (< P / 2), so the groups
        // stay ordered and every segment lies inside one group. Only while a
        // move costs a CTA at most 1/16 of its share: B96 S<=256 Hq32/Hkv16
        // (47 tiles per CTA, segments up to 8) was 2 us slower snapped, B128
        // S<=256 MHA (235 tiles per CTA, segments up to 16) 0.9 us faster.
        const int nseg = p.Hkv * p.QC;
        auto snap = [&](long long at) -> int {
          if (at >= U) return U;
          const int u = static_cast<int>(at);
          const int b = find_row(cum, p.B, u);
          const int base = cum[b];
          const int nt = (cum[b + 1] - base) / nseg;
          const int lo = base + (u - base) / nt * nt;
          return (u - lo <= lo + nt - u) ? lo : lo + nt;
        };
        rg.gr0 = snap(static_cast<long long>(rg.g) * P);
        rg.gr1 = snap(static_cast<long long>(rg.g + 1) * P);
        rg.Pw = max(1, (rg.gr1 - rg.gr0 + NW - 1) / NW);
        rg.wr0 = min(rg.gr1, rg.gr0 + rg.gi * rg.Pw);
        rg.wr1 = min(rg.gr1, rg.wr0 + rg.Pw);
      }
    }
    n_tiles = rg.wr1 - rg.wr0;
  } else {
    const int total = p.B * p.Hkv * p.QC * p.ns;
    if (wid >= total) return;
    w.s = wid % p.ns;
    const int rs = wid / p.ns;
    const int seg = rs % (p.Hkv * p.QC);
    w.b = rs / (p.Hkv * p.QC);
    w.kvh = seg / p.QC;
    w.qc = seg - w.kvh * p.QC;
    bool bad = false;
    const int S = p.seq_lens ? clamp_len(p, __ldg(p.seq_lens + w.b), bad) : p.seq_len;
    if (bad && w.s == 0 && seg == 0) flag(p, PA_STATUS_BAD_SEQLEN);
    const int ss = (S + p.ns - 1) / p.ns;       // torch_kernel.py:30
    w.t0 = w.s * ss;
    w.t1 = min(w.t0 + ss, S);
    w.tl0 = w.t0 / TILE;
    w.n = (w.t0 < w.t1) ? ((w.t1 - 1) / TILE - w.tl0 + 1) : 0;
    n_tiles = w.n;
  }
  // range of this warp's units (balanced) or of its split's tile ordinals
  const int range0 = (!kSplit) ? rg.wr0 : 0;
  const int range1 = (!kSplit) ? rg.wr1 : w.n;

  const uint32_t stage0 = smem_u32(smem + warp * NS * C::kStage);
  const uint32_t bar0 = smem_u32(&bars[warp * NS]);
  int* desc0 = descs + warp * NS * kDescInts;

  // Split schedule, empty split (split_kv_kernel.py:32-33): the partial LSE keeps
  // the sentinel; the last arriving split of the segment merges.
  if (kSplit && w.n == 0) {
    const int gc = min(8, G - w.qc * 8);
    for (int j = 0; j < gc; ++j) {
      const int hq = w.kvh * G + w.qc * 8 + j;
      const long long row = (static_cast<long long>(w.b) * p.Hq + hq) * p.ns + w.s;
      for (int d = lane; d < D; d += 32) p.o_part[row * D + d] = 0.f;
      if (lane == 0) p.lse_part[row] = kSentinel;
    }
    const int cid = (w.b * p.Hkv + w.kvh) * p.QC + w.qc;
    if (!arrive_elect_last<true>(p.counters + cid, p.ns, lane)) return;
    merge_splits<T, D>(p, w.b, w.kvh, w.qc, gc, lane);
    if (lane == 0) atomicExch(p.counters + cid, 0);
    return;
  }

  // ---- issuer: page batches of <= 32 boxes, current (pg_c) and next (pg_n)
  int u0c = range0, u1c = min(range1, range0 + bt_tiles);
  int u0n = u1c, u1n = min(range1, u1c + bt_tiles);
  int pg_c = INT_MIN, sl_c = 0, pg_n = INT_MIN, sl_n = 0;
  if (u0c < u1c) batch_pages<TILE, kSplit, kCum>(p, cum, rg, w, u0c, u1c, lane, pg_c, sl_c);
  Cursor ic;
  ic.b = w.b;
  ic.kvh = w.kvh;
  ic.qc = w.qc;
  ic.tile = w.tl0;
  ic.nt = ic.S = ic.seg_lo = 0;
  if (!kSplit && n_tiles > 0) decode_unit<TILE, kCum>(ic, p, cum, range0);
  int ord = 0;          // tile ordinal within the current batch
  int issued = 0;

  auto issue = [&](int st) {
    int t0, t1, fl;
    if (!kSplit) {
      piece_of<TILE>(ic, rg, t0, t1, fl);
    } else {
      const int k = u0c + ord;
      t0 = w.t0;
      t1 = w.t1;
      fl = (k == 0 ? kFirst : 0) | (k == w.n - 1 ? kLast : 0);
    }
    const int gc = min(8, G - ic.qc * 8);
    const int src = (ord << p.lspt) + (lane & spt_mask);
    const int phys = __shfl_sync(kFull, pg_c, src);
    const int pslot = __shfl_sync(kFull, sl_c, src);
    bool valid = lane <= spt_mask && phys != INT_MIN;
    if (valid && (phys < 0 || phys >= p.NB)) {
      flag(p, PA_STATUS_BAD_BLOCK);
      valid = false;
    }
    const unsigned vm = __ballot_sync(kFull, valid);
    const uint32_t bar = bar0 + st * 8;
    const uint32_t sk = stage0 + st * C::kStage;
    const bool first = fl & kFirst;
    if (lane == 0) {
      int* d = desc0 + st * kDescInts;
      reinterpret_cast<int4*>(d)[0] = make_int4(ic.b, ic.kvh, ic.qc, ic.tile * TILE);
      reinterpret_cast<int4*>(d)[1] = make_int4(t0, t1, ic.seg_lo, ic.seg_lo + ic.nt);
      reinterpret_cast<int4*>(d)[2] = make_int4(fl, gc, 0, 0);
      // per box: K and V, D/64 chunks of R rows x 128 B each; plus the query rows
      mbar_expect_tx(bar, __popc(vm) * 2 * H::kChunks * p.R * 128 + (first ? gc * D * 2 : 0));
    }
    __syncwarp();
    if (valid) {
      const uint32_t hs = p.R * 128;                     // one chunk of one box
      const uint32_t dk = sk + lane * H::kChunks * hs;   // this lane's box
      tma_load_5d(dk, &tmK, 0, pslot, 0, ic.kvh, phys, bar);
      tma_load_5d(dk + C::kKV, &tmV, 0, pslot, 0, ic.kvh, phys, bar);
    }
    if (first && lane < gc) {
      const int hq = ic.kvh * G + ic.qc * 8 + lane;
      bulk_load(sk + 2 * C::kKV + lane * D * 2, p.q + ic.b * p.q_sb + hq * p.q_sh, D * 2, bar);
    }
    ++issued;
    // advance to the next tile
    if (!kSplit) cursor_next<TILE, kCum>(ic, p); else ++ic.tile;
    if (u0c + ++ord < u1c) return;
    u0c = u0n;
    u1c = u1n;
    pg_c = pg_n;
    sl_c = sl_n;
    ord = 0;
    u0n = u1c;
    u1n = min(range1, u1c + bt_tiles);
    if (u0n < u1n) batch_pages<TILE, kSplit, kCum>(p, cum, rg, w, u0n, u1n, lane, pg_n, sl_n);
  };

  for (int s = 0; s < NS && issued < n_tiles; ++s) issue(s);
  // The second batch's block-table loads leave the path to the first copies: a
  // batch holds at least 8 tiles (32 boxes of >= 8 rows), more than the NS
  // issued above, so those never reached it (a range that ended inside the
  // first batch has no second one).
  if (u0n < u1n) batch_pages<TILE, kSplit, kCum>(p, cum, rg, w, u0n, u1n, lane, pg_n, sl_n);
  if (!kSplit) __syncthreads();   // gcnt is zero for every warp's merges
  if constexpr (kClu) asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
  // The next kernel in the stream may start its own prologue on SMs this grid
  // leaves; it waits for this grid's completion before touching memory.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // Zero-length rows, while the first copies are in flight.
  if (!kSplit && p.zero_rows)
    zero_length_rows<D, kCum>(p.B, p.Hq, p.out, p.o_sb, p.o_sh, p.lse, cum, p.seq_len);

  // ---- consumer state
  uint32_t qf[H::kSteps][2];
  float acc[H::kSteps][4];
  float m_run[2], l_run[2];
  uint32_t phase = 0;
  uint32_t mask_hi = 0, mask_lo = 0;   // which 16-bit halves carry hi / lo of p
  const int qd = lane & 3;             // column pair: columns 2*qd, 2*qd+1
  const int rr = lane >> 2;            // fragment row
  const float scl = p.scale_log2;

  // ldmatrix lane offsets in the box-major, 128-byte-swizzled tile: token row r
  // sits at r*128 + (r/R)*R*128*(D/64 - 1) (box start plus the other chunks of
  // earlier boxes), 16-byte piece c of a chunk at ((c ^ (r & 7)) << 4), chunk q
  // at +q*R*128.
  const uint32_t hs = p.R * 128;
  uint32_t offk[kMB], offv[kMB], swzk[4], swzv[4];
  {
    const int x = lane & 7;
    const int rk = ((lane >> 3) & 1) * 8 + x, yk = (lane >> 4) ^ x;
    const int rv = (lane >> 4) * 8 + x, yv = ((lane >> 3) & 1) ^ x;
#pragma unroll
    for (int mb = 0; mb < kMB; ++mb) {
      const int r1 = mb * 16 + rk, r2 = mb * 16 + rv;
      offk[mb] = r1 * 128 + ((r1 >> p.lR) << p.lR) * 128 * (H::kChunks - 1);
      offv[mb] = r2 * 128 + ((r2 >> p.lR) << p.lR) * 128 * (H::kChunks - 1);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      swzk[j] = ((2 * j) ^ yk) << 4;
      swzv[j] = ((2 * j) ^ yv) << 4;
    }
  }

  // A piece that crosses groups is published in two steps. Its arrival (an
  // acquire-release atomic through L2) goes out once the warp has no copy left
  // to issue: mid-stream, the round trip under a saturated DRAM (several us)
  // would hold back the warp's remaining tiles, while after the last issue it
  // overlaps the copies still in flight. The merge, for the last arriver, runs
  // after the warp's last tile, when none of the stream's registers are live
  // (one copy of the merge code, and no register pressure on the hot loop).
  int npend = 0, narr = 0;     // pending publishes; how many have arrived
  unsigned merge_mask = 0;     // pending entries this warp arrived last on
  auto pend_counter = [&](const int* r) {
    return p.counters + (r[0] * p.Hkv + r[1]) * p.QC + r[2];
  };
  auto arrive_pending = [&]() {
    // every arrival not yet made goes out before any result is awaited
    const int(*rec)[6] = pend_rec[kSplit ? 0 : warp];
    int old0 = 0, old1 = 0;
    __syncwarp();
    if (lane == 0) {
      if (narr == 0)
        asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;"
                     : "=r"(old0) : "l"(pend_counter(rec[0])) : "memory");
      if (npend > 1)
        asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;"
                     : "=r"(old1) : "l"(pend_counter(rec[1])) : "memory");
    }
    old0 = __shfl_sync(kFull, old0, 0);
    old1 = __shfl_sync(kFull, old1, 0);
    __syncwarp();
    for (int k = narr; k < npend; ++k) {
      const int* r = rec[k];
      const int n = (r[5] - 1) / rg.P - r[4] / rg.P + 1;
      if ((k == 0 ? old0 : old1) == n - 1) merge_mask |= 1u << k;
    }
    narr = npend;
  };
  // A group has at most two pieces that cross its boundaries (the segments
  // holding its first and its last unit), and one warp publishes each, so a
  // warp never holds more than two.
  auto defer_publish = [&](int b, int kvh, int qc, int gc, int seg_lo, int seg_hi) {
    if (lane == 0) {
      int* r = pend_rec[kSplit ? 0 : warp][npend];
      r[0] = b;
      r[1] = kvh;
      r[2] = qc;
      r[3] = gc;
      r[4] = seg_lo;
      r[5] = seg_hi;
    }
    __syncwarp();
    ++npend;
  };

  int st = 0;
  for (int i = 0; i < n_tiles; ++i) {
    if (!kSplit && narr < npend && issued == n_tiles) arrive_pending();
    const uint32_t sk = stage0 + st * C::kStage;
    const uint32_t sv = sk + C::kKV;
    const uint32_t sq = sk + 2 * C::kKV;

    if (!mbar_wait(bar0 + st * 8, (phase >> st) & 1)) {
      drain_after_timeout<NS>(p.status, bar0, st, phase, issued - i - 1);
      if (kClu) break;   // rank 0's merging warps still wait (bounded) for every push
      return;
    }
    phase ^= 1u << st;
    const int* d = desc0 + st * kDescInts;
    const int4 d0 = reinterpret_cast<const int4*>(d)[0];
    const int4 d1 = reinterpret_cast<const int4*>(d)[1];
    const int4 d2 = reinterpret_cast<const int4*>(d)[2];
    const int tb = d0.w, t0 = d1.x, t1 = d1.y, fl = d2.x, gc = d2.y;

    if (fl & kFirst) {
      // Query fragments (B operand of S^T = K Q^T): column n -> query head.
      const int n = rr;
      const int head = kDup ? (n < 2 * gc ? (n < gc ? n : n - gc) : -1) : (n < gc ? n : -1);
#pragma unroll
      for (int ks = 0; ks < H::kSteps; ++ks) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t v = 0;
          if (head >= 0) {
            const uint32_t addr = sq + head * D * 2 + (ks * 16 + h * 8 + qd * 2) * 2;
            asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
          }
          qf[ks][h] = v;
        }
      }
#pragma unroll
      for (int md = 0; md < H::kSteps; ++md)
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[md][r] = 0.f;
      m_run[0] = m_run[1] = -INFINITY;
      l_run[0] = l_run[1] = 0.f;
      const int c0 = 2 * qd, c1 = c0 + 1;
      mask_hi = (c0 < gc ? 0x0000ffffu : 0u) | (c1 < gc ? 0xffff0000u : 0u);
      if (kDup) {
        mask_lo = ((c0 >= gc && c0 < 2 * gc) ? 0x0000ffffu : 0u) |
                  ((c1 >= gc && c1 < 2 * gc) ? 0xffff0000u : 0u);
      } else {
        mask_lo = mask_hi;
      }
    }

    // ---- S^T = K Q^T: TILE tokens x 8 query columns, FP32 accumulate.
    float s[kMB][4];
#pragma unroll
    for (int mb = 0; mb < kMB; ++mb) {
#pragma unroll
      for (int r = 0; r < 4; ++r) s[mb][r] = 0.f;
#pragma unroll
      for (int ks = 0; ks < H::kSteps; ++ks) {
        uint32_t a[4];
        ldsm_x4(sk + offk[mb] + (ks >> 2) * hs + swzk[ks & 3], a);
        Mma<T>::run(s[mb], a, qf[ks][0], qf[ks][1]);
      }
    }

    // ---- mask, online softmax (split_kv_kernel.py:68-77); scores kept unscaled,
    // the scale is folded into the exponent.
    const bool partial = (t0 > tb) || (t1 < tb + TILE);
    if (partial) {
#pragma unroll
      for (int mb = 0; mb < kMB; ++mb)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int tok = tb + mb * 16 + rr + (r >> 1) * 8;
          if (tok < t0 || tok >= t1) s[mb][r] = -INFINITY;
        }
    }
    float alpha[2], mneg[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float mx = fmaxf(s[0][e], s[0][e + 2]);
#pragma unroll
      for (int mb = 1; mb < kMB; ++mb) mx = fmaxf(mx, fmaxf(s[mb][e], s[mb][e + 2]));
      mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 4));
      mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 16));
      const float mn = fmaxf(m_run[e], mx);
      alpha[e] = exp2f((m_run[e] - mn) * scl);
      m_run[e] = mn;
      mneg[e] = -mn * scl;
    }
    float psum[2] = {0.f, 0.f};
#pragma unroll
    for (int mb = 0; mb < kMB; ++mb)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const float pv = exp2f(fmaf(s[mb][r], scl, mneg[r & 1]));
        s[mb][r] = pv;
        psum[r & 1] += pv;
      }
    l_run[0] = fmaf(l_run[0], alpha[0], psum[0]);
    l_run[1] = fmaf(l_run[1], alpha[1], psum[1]);
    if (__any_sync(kFull, (alpha[0] != 1.f) || (alpha[1] != 1.f))) {
#pragma unroll
      for (int md = 0; md < H::kSteps; ++md) {
        acc[md][0] *= alpha[0];
        acc[md][1] *= alpha[1];
        acc[md][2] *= alpha[0];
        acc[md][3] *= alpha[1];
      }
    }

    // ---- P^T as the B operand; hi + lo keeps ~16 (bf16) / 22 (fp16) bits of p.
    uint32_t bh[kMB][2], bl[kMB][2];
#pragma unroll
    for (int kb = 0; kb < kMB; ++kb) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t hi, lo;
        Mma<T>::split2(s[kb][half * 2], s[kb][half * 2 + 1], hi, lo);
        if (kDup) {
          bh[kb][half] = movm_trans((hi & mask_hi) | (lo & mask_lo));
        } else {
          bh[kb][half] = movm_trans(hi & mask_hi);
          bl[kb][half] = movm_trans(lo & mask_lo);
        }
      }
    }

    // ---- O^T += V^T P^T (dims x columns).
#pragma unroll
    for (int kb = 0; kb < kMB; ++kb) {
      uint32_t m01 = 0xffffffffu, m23 = 0xffffffffu;
      if (partial) {
        const int tk = tb + kb * 16 + qd * 2;
        m01 = ((tk >= t0 && tk < t1) ? 0x0000ffffu : 0u) |
              ((tk + 1 >= t0 && tk + 1 < t1) ? 0xffff0000u : 0u);
        m23 = ((tk + 8 >= t0 && tk + 8 < t1) ? 0x0000ffffu : 0u) |
              ((tk + 9 >= t0 && tk + 9 < t1) ? 0xffff0000u : 0u);
      }
#pragma unroll
      for (int md = 0; md < H::kSteps; ++md) {
        uint32_t a[4];
        ldsm_x4_t(sv + offv[kb] + (md >> 2) * hs + swzv[md & 3], a);
        if (partial) {
          a[0] &= m01;
          a[1] &= m01;
          a[2] &= m23;
          a[3] &= m23;
        }
        Mma<T>::run(acc[md], a, bh[kb][0], bh[kb][1]);
        if (!kDup) Mma<T>::run(acc[md], a, bl[kb][0], bl[kb][1]);
      }
    }

    __syncwarp();
    const int cur = st;
    st = (st + 1 == NS) ? 0 : st + 1;
    if (issued < n_tiles) issue(cur);

    if (!(fl & kLast)) continue;

    // ---------------------------------------------------------- piece epilogue
    const int b = d0.x, kvh = d0.y, qc = d0.z;
    const int seg_lo = d1.z, seg_hi = d1.w;
    float lsum[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float v = l_run[e];
      v += __shfl_xor_sync(kFull, v, 4);
      v += __shfl_xor_sync(kFull, v, 8);
      v += __shfl_xor_sync(kFull, v, 16);
      lsum[e] = v;
    }
    // Dup layout: column c + gc holds the low part of column c.
    float o[H::kSteps][4];
#pragma unroll
    for (int md = 0; md < H::kSteps; ++md)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        float v = acc[md][r];
        if (kDup) {
          const float partner =
              (gc == 1) ? acc[md][r | 1] : __shfl_down_sync(kFull, v, gc >> 1);
          v += partner;
        }
        o[md][r] = v;
      }

    // Where this warp's piece goes: 0 final output, 1 the group's global slot
    // (or the split's row), 2 this warp's shared-memory slot.
    const int dest = (kSplit) ? 1 : (fl & kWarpSeg) ? 0 : (fl & kWarpGroup) ? 1 : 2;
    const int glo = max(seg_lo, rg.gr0), ghi = min(seg_hi, rg.gr1);
    const long long gslot = 2ll * rg.g + (glo == rg.gr0 ? 0 : 1);
    const int wside = (max(seg_lo, rg.wr0) == rg.wr0) ? 0 : 1;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int c = qd * 2 + e;
      if (c >= gc) continue;
      const int hq = kvh * G + qc * 8 + c;
      const float lv = fmaxf(lsum[e], 1e-20f);
      const float inv_l = __fdividef(1.f, lv);
      const float lse = (m_run[e] * scl + __log2f(lv)) * kLn2;
      if (dest == 0) {
        char* dst = p.out + b * p.o_sb + hq * p.o_sh;
#pragma unroll
        for (int md = 0; md < H::kSteps; ++md) {
          const int d0i = md * 16 + rr;
          *reinterpret_cast<uint16_t*>(dst + d0i * 2) = Mma<T>::from_float(o[md][e] * inv_l);
          *reinterpret_cast<uint16_t*>(dst + (d0i + 8) * 2) =
              Mma<T>::from_float(o[md][e + 2] * inv_l);
        }
        if (rr == 0 && p.lse) p.lse[b * p.Hq + hq] = lse;
      } else if (kClu && dest == 1) {
        // the CTA's piece, straight into rank 0's shared memory
        const uint32_t r =
            cluster_map(smem_u32(cslot + (crank * p.slot_cols + c) * H::kSlotStride), 0);
#pragma unroll
        for (int md = 0; md < H::kSteps; ++md) {
          const int d0i = md * 16 + rr;
          st_cluster(r + d0i * 4, o[md][e] * inv_l);
          st_cluster(r + (d0i + 8) * 4, o[md][e + 2] * inv_l);
        }
        if (rr == 0) st_cluster(r + D * 4, lse);
      } else {
        float* od;
        float* ld;
        if (dest == 2) {
          od = gslots + ((rg.gi * 2 + wside) * p.slot_cols + c) * H::kSlotStride;
          ld = od + D;
        } else if (!kSplit) {
          od = gslot_row<D>(p, gslot, c);
          ld = gslot_lse(p, gslot, c);
        } else {
          const long long row = (static_cast<long long>(b) * p.Hq + hq) * p.ns + w.s;
          od = p.o_part + row * D;
          ld = p.lse_part + row;
        }
#pragma unroll
        for (int md = 0; md < H::kSteps; ++md) {
          const int d0i = md * 16 + rr;
          od[d0i] = o[md][e] * inv_l;
          od[d0i + 8] = o[md][e + 2] * inv_l;
        }
        if (rr == 0) *ld = lse;
      }
    }
    if (dest == 0) continue;

    if (kSplit) {
      // split schedule: the last split of the segment merges all ns rows
      const int cid = (b * p.Hkv + kvh) * p.QC + qc;
      if (!arrive_elect_last<true>(p.counters + cid, p.ns, lane)) continue;
      merge_splits<T, D>(p, b, kvh, qc, gc, lane);
      if (lane == 0) atomicExch(p.counters + cid, 0);
      continue;
    }
    if (dest == 1) {
      if constexpr (kClu)
        mbar_arrive_cluster(cluster_map(cbar, 0));
      else if (!p.post_merge)
        defer_publish(b, kvh, qc, gc, seg_lo, seg_hi);
      continue;
    }

    // Shared-memory piece: the group's last warp on this piece merges the
    // warps' rows into the group's piece.
    const int w_first = (glo - rg.gr0) / rg.Pw;
    const int nw = (ghi - 1 - rg.gr0) / rg.Pw - w_first + 1;
    if (!arrive_elect_last<false>(gcnt + w_first, nw, lane)) continue;
    if (lane == 0) gcnt[w_first] = 0;
    for (int j = 0; j < gc; ++j) {
      auto src = [&](int k, const float*& row, const float*& lp) {
        const int wk = w_first + k;
        const int start = rg.gr0 + wk * rg.Pw;
        const int side = (max(glo, start) == start) ? 0 : 1;
        row = gslots + ((wk * 2 + side) * p.slot_cols + j) * H::kSlotStride;
        lp = row + D;
      };
      RowV<H::kLaneF> o4;
      float lse;
      merge_rows_smem<D>(nw, lane, src, o4, lse);
      if (fl & kGroupSeg) {
        store_out<T, D>(p, b, kvh * G + qc * 8 + j, lane, o4, lse);
      } else if (kClu) {
        const uint32_t r =
            cluster_map(smem_u32(cslot + (crank * p.slot_cols + j) * H::kSlotStride), 0);
#pragma unroll
        for (int i = 0; i < H::kLaneF; ++i) st_cluster(r + (lane * H::kLaneF + i) * 4, o4.f[i]);
        if (lane == 0) st_cluster(r + D * 4, lse);
      } else {
        store_row(gslot_row<D>(p, gslot, j), lane, o4);
        if (lane == 0) *gslot_lse(p, gslot, j) = lse;
      }
    }
    if constexpr (kClu)
      mbar_arrive_cluster(cluster_map(cbar, 0));
    else if (!(fl & kGroupSeg) && !p.post_merge)
      defer_publish(b, kvh, qc, gc, seg_lo, seg_hi);
  }
  if (!kSplit && npend > 0) {
    if (narr < npend) arrive_pending();
    for (int k = 0; k < npend; ++k) {
      if (!(merge_mask & (1u << k))) continue;
      const int* r = pend_rec[kSplit ? 0 : warp][k];
      merge_groups<T, D>(p, rg, r[0], r[1], r[2], r[3], r[4], r[5], lane);
      if (lane == 0) atomicExch(pend_counter(r), 0);
    }
  }
  if constexpr (kClu) {
    // Rank 0 stays resident until every CTA's piece has landed in its shared
    // memory (the other CTAs only write there and may exit at once).
    if (crank == 0) merge_cluster<T, D, NW>(p, cslot, cbar, static_cast<int>(cid), warp, lane);
  }
}

#if PA_HOST_PART
// ----------------------------------------------------------------------------
// ----------------------------------------------------------------------------
// KV-cache append: one thread per 16-byte chunk of a K or V row
// ----------------------------------------------------------------------------
struct AppendParams {
  const char* key;
  const char* value;
  long long k_st, k_sh, v_st, v_sh;          // bytes
  char* kc;
  char* vc;
  long long kc_sb, kc_ss, kc_sh, vc_sb, vc_ss, vc_sh;   // bytes
  const long long* slots;
  int T, Hkv, chunks, bs, NB;                // chunks: 16-byte pieces per row
  unsigned* status;
};

__global__ void __launch_bounds__(256) cache_append_kernel(const AppendParams a) {
  const long long per_tok = 2ll * a.Hkv * a.chunks;
  const long long total = per_tok * a.T;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(i / per_tok);
    long long r = i - t * per_tok;
    const int is_v = static_cast<int>(r / (static_cast<long long>(a.Hkv) * a.chunks));
    r -= static_cast<long long>(is_v) * a.Hkv * a.chunks;
    const int h = static_cast<int>(r / a.chunks);
    const int c = static_cast<int>(r - static_cast<long long>(h) * a.chunks);
    const long long slot = __ldg(a.slots + t);
    if (slot < 0) continue;
    const long long blk = slot / a.bs;
    const int off = static_cast<int>(slot - blk * a.bs);
    if (blk >= a.NB) {
      if (a.status && c == 0 && h == 0 && !is_v) atomicOr(a.status, PA_STATUS_BAD_BLOCK);
      continue;
    }
    const char* src = is_v ? a.value + t * a.v_st + h * a.v_sh : a.key + t * a.k_st + h * a.k_sh;
    char* dst = is_v ? a.vc + blk * a.vc_sb + off * a.vc_ss + h * a.vc_sh
                     : a.kc + blk * a.kc_sb + off * a.kc_ss + h * a.kc_sh;
    reinterpret_cast<uint4*>(dst)[c] = __ldg(reinterpret_cast<const uint4*>(src) + c);
  }
}

// ----------------------------------------------------------------------------
// Cross-group merge pass (balanced schedule)
// ----------------------------------------------------------------------------
// When few segments each span many groups, every group finishes at about the
// same time and the in-kernel merge (the last group's one warp walking gc
// columns x n pieces, an L2 round trip per column and per 8 pieces) is the
// step's tail. This kernel follows the decode kernel in the stream instead
// (programmatic dependent launch): one CTA per segment that crosses a group
// boundary, its eight warps split over the segment's columns and, for fewer
// columns, over its pieces; each lane keeps 64 floats of pieces in flight.
// Same arithmetic as merge_rows (split_kv_kernel.py:101-122): pieces with
// LSE <= -1e29 are skipped and the sum is clamped at 1e-20.
struct MergeParams {
  const float* o_part;      // group slots [2 * groups][slot_cols][D]
  const float* lse_part;    // [2 * groups][slot_cols]
  char* out;
  long long o_sb, o_sh;     // bytes
  float* lse;
  const int* seq_lens;      // per-row lengths (kCum), clamped to [0, cap]
  int cap;
  int B, Hkv, G, QC, slot_cols;
  int tile;                 // tokens per unit
  int ngroups, gsz;
  int U, P, nt_u, per_row;  // same-length rows; P: units per group
  int by_segment;           // 1: block x is a segment, 0: block x + 1 is a group boundary
  int col_split;            // 1: block y is one query column (segments of many pieces)
};

template <typename T, int D, bool kCum>
__global__ void __launch_bounds__(256) merge_segments_kernel(const MergeParams m) {
  constexpr int N = HD<D>::kLaneF;
  constexpr int kRows = 64 / N;   // pieces in flight per lane
  __shared__ __align__(16) float s_acc[8][D];
  __shared__ float s_ml[8][2];
  __shared__ int s_cum[kCum ? kCumMax + 1 : 1];
  __shared__ int s_tot[8];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // The decode kernel's partials are complete and visible after the wait.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  const int nseg = m.Hkv * m.QC;   // segments per row
  int U = m.U, P = m.P;
  if constexpr (kCum) {
    // Per-row unit prefix sums, formed as the decode kernel forms them.
    const int chunk = (m.B + 255) / 256;
    const int lo = min(m.B, static_cast<int>(threadIdx.x) * chunk);
    const int hi = min(m.B, lo + chunk);
    int local = 0;
    for (int b = lo; b < hi; ++b) {
      const int S = min(max(__ldg(m.seq_lens + b), 0), m.cap);
      local += nseg * ((S + m.tile - 1) / m.tile);
    }
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) s_tot[warp] = incl;
    __syncthreads();
    int run = incl - local;
    for (int k = 0; k < warp; ++k) run += s_tot[k];
    for (int b = lo; b < hi; ++b) {
      s_cum[b] = run;
      const int S = min(max(__ldg(m.seq_lens + b), 0), m.cap);
      run += nseg * ((S + m.tile - 1) / m.tile);
    }
    if (threadIdx.x == 255) s_cum[m.B] = run;
    __syncthreads();
    U = s_cum[m.B];
    P = max((U + m.ngroups - 1) / m.ngroups, m.gsz);
  }

  // The segment: units [seg_lo, seg_lo + nt) of row b, segment index seg.
  int b, seg, seg_lo, nt;
  if (m.by_segment) {
    b = blockIdx.x / nseg;
    seg = blockIdx.x - b * nseg;
    if constexpr (kCum) {
      const int S = min(max(__ldg(m.seq_lens + b), 0), m.cap);
      nt = (S + m.tile - 1) / m.tile;
      seg_lo = s_cum[b] + seg * nt;
    } else {
      nt = m.nt_u;
      seg_lo = b * m.per_row + seg * nt;
    }
    if (nt == 0 || seg_lo / P == (seg_lo + nt - 1) / P) return;   // inside one group
  } else {
    const long long u64 = static_cast<long long>(blockIdx.x + 1) * P;
    if (u64 >= U) return;
    const int u = static_cast<int>(u64);
    int row_base;
    if constexpr (kCum) {
      b = find_row(s_cum, m.B, u);
      row_base = s_cum[b];
      const int S = min(max(__ldg(m.seq_lens + b), 0), m.cap);
      nt = (S + m.tile - 1) / m.tile;
    } else {
      b = u / m.per_row;
      row_base = b * m.per_row;
      nt = m.nt_u;
    }
    seg = (u - row_base) / nt;
    seg_lo = row_base + seg * nt;
    // Only the segment's first crossing merges it.
    if (seg_lo == u || seg_lo / P != static_cast<int>(blockIdx.x)) return;
  }
  const int seg_hi = seg_lo + nt;
  const int g_first = seg_lo / P;
  const int n = (seg_hi - 1) / P - g_first + 1;
  const int kvh = seg / m.QC;
  const int qc = seg - kvh * m.QC;
  int gc = min(8, m.G - qc * 8);
  int j0 = 0;                       // first column of this CTA
  if (m.col_split) {
    j0 = blockIdx.y;
    if (j0 >= gc) return;
    gc = 1;                         // columns of this CTA
  }
  const int wpc = 8 / gc;           // warps per column
  const int jl = warp / wpc;        // column of this warp, within the CTA's
  const int r = warp - jl * wpc;    // this warp's pieces: r, r + wpc, ...
  const int j = j0 + jl;

  float mx = kValidLse, sum = 0.f;
  RowV<N> acc;
#pragma unroll
  for (int i = 0; i < N; ++i) acc.f[i] = 0.f;
  if (jl < gc) {
    for (int k0 = r; k0 < n; k0 += kRows * wpc) {
      float l[kRows];
      RowV<N> v[kRows];
#pragma unroll
      for (int t = 0; t < kRows; ++t) {
        const int k = k0 + t * wpc;
        if (k < n) {
          const int g = g_first + k;
          const long long sl = 2ll * g + (max(seg_lo, g * P) == g * P ? 0 : 1);
          l[t] = __ldcg(m.lse_part + sl * m.slot_cols + j);
          v[t] = load_row<true, N>(m.o_part + (sl * m.slot_cols + j) * D, lane);
        } else {
          l[t] = kSentinel;
#pragma unroll
          for (int i = 0; i < N; ++i) v[t].f[i] = 0.f;
        }
      }
      float bm = mx;
#pragma unroll
      for (int t = 0; t < kRows; ++t)
        if (l[t] > kValidLse) bm = fmaxf(bm, l[t]);
      const float f = exp2f((mx - bm) * kLog2e);
      sum *= f;
#pragma unroll
      for (int i = 0; i < N; ++i) acc.f[i] *= f;
#pragma unroll
      for (int t = 0; t < kRows; ++t) {
        const float wgt = (l[t] > kValidLse) ? exp2f((l[t] - bm) * kLog2e) : 0.f;
        sum += wgt;
#pragma unroll
        for (int i = 0; i < N; ++i) acc.f[i] = fmaf(wgt, v[t].f[i], acc.f[i]);
      }
      mx = bm;
    }
  }
  if (wpc > 1) {   // the column's warps meet in shared memory
    if (jl < gc) {
      store_row(&s_acc[warp][0], lane, acc);
      if (lane == 0) {
        s_ml[warp][0] = mx;
        s_ml[warp][1] = sum;
      }
    }
    __syncthreads();
    if (jl < gc && r == 0) {
      float M = kValidLse;
      for (int i = 0; i < wpc; ++i) M = fmaxf(M, s_ml[warp + i][0]);
      sum = 0.f;
#pragma unroll
      for (int i = 0; i < N; ++i) acc.f[i] = 0.f;
      for (int w2 = 0; w2 < wpc; ++w2) {
        const float f = exp2f((s_ml[warp + w2][0] - M) * kLog2e);
        sum = fmaf(s_ml[warp + w2][1], f, sum);
        const RowV<N> a2 = load_row<false, N>(&s_acc[warp + w2][0], lane);
#pragma unroll
        for (int i = 0; i < N; ++i) acc.f[i] = fmaf(f, a2.f[i], acc.f[i]);
      }
      mx = M;
    }
  }
  if (jl >= gc || r != 0) return;
  const float inv = 1.f / fmaxf(sum, 1e-20f);
  const int hq = kvh * m.G + qc * 8 + j;
  char* dst = m.out + b * m.o_sb + hq * m.o_sh + lane * N * 2;
  uint32_t w[N / 2];
#pragma unroll
  for (int i = 0; i < N / 2; ++i)
    w[i] = pack16(Mma<T>::from_float(acc.f[2 * i] * inv),
                  Mma<T>::from_float(acc.f[2 * i + 1] * inv));
  if constexpr (N == 2) {
    *reinterpret_cast<uint32_t*>(dst) = w[0];
  } else if constexpr (N == 4) {
    *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
  } else {
    *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  if (lane == 0 && m.lse) m.lse[b * m.G * m.Hkv + hq] = sum > 0.f ? mx + logf(sum) : kSentinel;
}

// ----------------------------------------------------------------------------
// Bandwidth probes (replace measure_peak_bw.py:15-21's Triton copy kernel)
// ----------------------------------------------------------------------------
// Each CTA copies one contiguous chunk of 256 threads x 8 x 16 B = 32 KB: all
// eight loads of a thread are issued before its stores, and the grid covers
// the buffer once (no grid-stride loop), so every SM keeps many independent
// chunks in flight. On B200 this copies at ~6.86 TB/s (read + write), above a
// device-to-device cudaMemcpy of the same buffer (~6.55 TB/s); a persistent
// grid-stride form with 4 loads per iteration reached ~5.9 TB/s.
constexpr int kCopyThreads = 256;
constexpr int kCopyUnroll = 8;

__global__ void __launch_bounds__(kCopyThreads) stream_copy_kernel(const uint4* __restrict__ src,
                                                                   uint4* __restrict__ dst,
                                                                   size_t n) {
  const size_t base = static_cast<size_t>(blockIdx.x) * kCopyThreads * kCopyUnroll + threadIdx.x;
  uint4 v[kCopyUnroll];
#pragma unroll
  for (int u = 0; u < kCopyUnroll; ++u) {
    const size_t k = base + static_cast<size_t>(u) * kCopyThreads;
    if (k < n) v[u] = src[k];
  }
#pragma unroll
  for (int u = 0; u < kCopyUnroll; ++u) {
    const size_t k = base + static_cast<size_t>(u) * kCopyThreads;
    if (k < n) dst[k] = v[u];
  }
}

__global__ void __launch_bounds__(512) stream_read_kernel(const uint4* __restrict__ src, size_t n,
                                                          uint32_t* sink) {
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  uint32_t x = 0;
  for (; i + 3 * stride < n; i += 4 * stride) {
    const uint4 a = __ldcs(src + i);
    const uint4 b = __ldcs(src + i + stride);
    const uint4 c = __ldcs(src + i + 2 * stride);
    const uint4 d = __ldcs(src + i + 3 * stride);
    x ^= a.x ^ a.y ^ a.z ^ a.w ^ b.x ^ b.y ^ b.z ^ b.w ^ c.x ^ c.y ^ c.z ^ c.w ^ d.x ^ d.y ^ d.z ^
         d.w;
  }
  for (; i < n; i += stride) {
    const uint4 a = __ldcs(src + i);
    x ^= a.x ^ a.y ^ a.z ^ a.w;
  }
  // One relaxed atomic per warp keeps the loads alive without a reduction tree.
  x ^= __shfl_xor_sync(kFull, x, 16);
  x ^= __shfl_xor_sync(kFull, x, 8);
  x ^= __shfl_xor_sync(kFull, x, 4);
  x ^= __shfl_xor_sync(kFull, x, 2);
  x ^= __shfl_xor_sync(kFull, x, 1);
  if ((threadIdx.x & 31) == 0 && x == 0x9e3779b9u) atomicXor(sink, x);
}

// ----------------------------------------------------------------------------
// CUDA-core path for the shapes the tile kernels do not cover
// ----------------------------------------------------------------------------
// head_dim 32, and pages of a size that is not a multiple of 8 tokens (1, 2,
// 4, ...; the reference accepts any power of two). The reference's own two
// stages on CUDA cores: one warp per (row, query head, split) walks its
// tokens 32 at a time -- lane j scores token j against the query (held in
// shared memory), then the lanes, each owning D/32 dimensions, accumulate
// p_j V_j (split_kv_kernel.py:12-84, FP32 partials); then one warp per (row,
// query head) merges the splits (split_kv_kernel.py:87-122). Partials are
// [B, Hq, ns, D] and [B, Hq, ns] fp32; an empty split stores LSE -1e30.
struct GenParams {
  const char* q;
  long long q_sb, q_sh;                     // bytes
  const char* kc;
  const char* vc;
  long long k_sb, k_ss, k_sh, v_sb, v_ss, v_sh;   // bytes
  const int* bt;
  long long bt_sb;                          // elements
  int max_blocks;
  const int* seq_lens;
  int seq_len;
  int B, Hq, G, bs, NB, ns;
  float scale_log2;
  float* o_part;
  float* lse_part;
  char* out;
  long long o_sb, o_sh;                     // bytes
  float* lse;
  unsigned* status;
};

template <typename T>
__device__ __forceinline__ float half_bits_to_float(uint16_t x);
template <>
__device__ __forceinline__ float half_bits_to_float<__half>(uint16_t x) {
  return __half2float(__ushort_as_half(x));
}
template <>
__device__ __forceinline__ float half_bits_to_float<__nv_bfloat16>(uint16_t x) {
  return __bfloat162float(__ushort_as_bfloat16(x));
}

// N consecutive 16-bit values at p (2N-byte aligned) as floats.
template <typename T, int N>
__device__ __forceinline__ void load_halfs(const char* p, float (&f)[N]) {
  uint16_t h[N];
  if constexpr (N == 1) {
    h[0] = *reinterpret_cast<const uint16_t*>(p);
  } else if constexpr (N == 2) {
    const uint32_t v = __ldg(reinterpret_cast<const unsigned int*>(p));
    h[0] = v & 0xffff; h[1] = v >> 16;
  } else if constexpr (N == 4) {
    const uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
    h[0] = v.x & 0xffff; h[1] = v.x >> 16; h[2] = v.y & 0xffff; h[3] = v.y >> 16;
  } else {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      h[2 * i] = w[i] & 0xffff;
      h[2 * i + 1] = w[i] >> 16;
    }
  }
#pragma unroll
  for (int i = 0; i < N; ++i) f[i] = half_bits_to_float<T>(h[i]);
}

template <typename T, int D>
__global__ void __launch_bounds__(128) generic_split_kernel(const GenParams g) {
  constexpr int N = D / 32;   // dimensions per lane in the PV product
  __shared__ float qs[4][D];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const long long w = static_cast<long long>(blockIdx.x) * 4 + warp;
  if (w >= static_cast<long long>(g.B) * g.Hq * g.ns) return;
  const int s = static_cast<int>(w % g.ns);
  const long long rowhq = w / g.ns;          // b * Hq + hq
  const int hq = static_cast<int>(rowhq % g.Hq);
  const int b = static_cast<int>(rowhq / g.Hq);
  const int kvh = hq / g.G;
  int S = g.seq_len;
  if (g.seq_lens) {
    const long long cap = static_cast<long long>(g.max_blocks) * g.bs;
    const int raw = __ldg(g.seq_lens + b);
    S = raw < 0 ? 0 : (raw > cap ? static_cast<int>(cap) : raw);
    if ((raw < 0 || raw > cap) && lane == 0 && s == 0 && hq == 0 && g.status)
      atomicOr(g.status, PA_STATUS_BAD_SEQLEN);
  }
  const int ss = (S + g.ns - 1) / g.ns;      // torch_kernel.py:30
  const int t0 = s * ss;
  const int t1 = min(t0 + ss, S);
  float* op = g.o_part + w * D;
  if (t0 >= t1) {                            // split_kv_kernel.py:32-33: the sentinel stays
    for (int d = lane; d < D; d += 32) op[d] = 0.f;
    if (lane == 0) g.lse_part[w] = kSentinel;
    return;
  }
  const uint16_t* qp = reinterpret_cast<const uint16_t*>(g.q + b * g.q_sb + hq * g.q_sh);
  for (int d = lane; d < D; d += 32) qs[warp][d] = half_bits_to_float<T>(qp[d]);
  __syncwarp();
  float m = -INFINITY, l = 0.f, acc[N];
#pragma unroll
  for (int i = 0; i < N; ++i) acc[i] = 0.f;
  for (int c = t0; c < t1; c += 32) {
    const int t = c + lane;
    int page = -1, slot = 0;
    if (t < t1) {                            // split_kv_kernel.py:52-58
      const int lb = t / g.bs;
      page = __ldg(g.bt + b * g.bt_sb + lb);
      slot = t - lb * g.bs;
      if (page < 0 || page >= g.NB) {
        if (g.status) atomicOr(g.status, PA_STATUS_BAD_BLOCK);
        page = -1;
      }
    }
    float sc = -INFINITY;                    // masked tokens score -inf (:68-69)
    if (page >= 0) {
      const char* kr = g.kc + page * g.k_sb + slot * g.k_ss + kvh * g.k_sh;
      float dot = 0.f;
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        float f[8];
        load_halfs<T, 8>(kr + i * 16, f);
#pragma unroll
        for (int e = 0; e < 8; ++e) dot = fmaf(f[e], qs[warp][i * 8 + e], dot);
      }
      sc = dot * g.scale_log2;
    }
    float cm = sc;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(kFull, cm, o));
    const float mn = fmaxf(m, cm);
    if (mn == -INFINITY) continue;           // every page of the step was out of range
    const float alpha = exp2f(m - mn);
    const float pv = (sc == -INFINITY) ? 0.f : exp2f(sc - mn);
    float ps = pv;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(kFull, ps, o);
    l = fmaf(l, alpha, ps);
#pragma unroll
    for (int i = 0; i < N; ++i) acc[i] *= alpha;
    m = mn;
    const int nj = min(32, t1 - c);
    for (int j = 0; j < nj; ++j) {
      const float pj = __shfl_sync(kFull, pv, j);
      const int pg = __shfl_sync(kFull, page, j);
      const int sl = __shfl_sync(kFull, slot, j);
      if (pg < 0) continue;
      float f[N];
      load_halfs<T, N>(g.vc + pg * g.v_sb + sl * g.v_ss + kvh * g.v_sh + lane * N * 2, f);
#pragma unroll
      for (int i = 0; i < N; ++i) acc[i] = fmaf(pj, f[i], acc[i]);
    }
  }
  // split_kv_kernel.py:79-84: normalised partial and its LSE (natural log)
  const float lv = fmaxf(l, 1e-20f);
#pragma unroll
  for (int i = 0; i < N; ++i) op[lane * N + i] = acc[i] / lv;
  if (lane == 0) g.lse_part[w] = (m == -INFINITY) ? kSentinel : (m + log2f(lv)) * kLn2;
}

template <typename T, int D>
__global__ void __launch_bounds__(128) generic_reduce_kernel(const GenParams g) {
  constexpr int N = D / 32;
  const int lane = threadIdx.x & 31;
  const long long w = static_cast<long long>(blockIdx.x) * 4 + (threadIdx.x >> 5);
  if (w >= static_cast<long long>(g.B) * g.Hq) return;
  const int hq = static_cast<int>(w % g.Hq);
  const int b = static_cast<int>(w / g.Hq);
  const float* lp = g.lse_part + w * g.ns;
  const float* op = g.o_part + w * g.ns * D;
  // split_kv_kernel.py:101-122: skip LSE <= -1e29, running max, divide by
  // max(sum, 1e-20)
  float gmax = kValidLse, gsum = 0.f, acc[N];
#pragma unroll
  for (int i = 0; i < N; ++i) acc[i] = 0.f;
  for (int s = 0; s < g.ns; ++s) {
    const float l = lp[s];
    if (l <= kValidLse) continue;
    const float mn = fmaxf(gmax, l);
    const float f = exp2f((gmax - mn) * kLog2e);
    const float wgt = exp2f((l - mn) * kLog2e);
    gsum = fmaf(gsum, f, wgt);
#pragma unroll
    for (int i = 0; i < N; ++i) acc[i] = fmaf(acc[i], f, wgt * op[s * D + lane * N + i]);
    gmax = mn;
  }
  const float inv = 1.f / fmaxf(gsum, 1e-20f);
  uint16_t* dst = reinterpret_cast<uint16_t*>(g.out + b * g.o_sb + hq * g.o_sh) + lane * N;
#pragma unroll
  for (int i = 0; i < N; ++i) dst[i] = Mma<T>::from_float(acc[i] * inv);
  if (lane == 0 && g.lse) g.lse[w] = gsum > 0.f ? gmax + logf(gsum) : kSentinel;
}

// ----------------------------------------------------------------------------
// Self-test of the bounded barrier wait
// ----------------------------------------------------------------------------
// The decode kernel's only device-side failure handling: a copy barrier that
// never completes its phase. One warp runs the same pieces on a two-stage
// ring: stage 0's barrier expects two arrivals and only one ever comes (no
// copy is attached to it), so its wait gives up after `limit_ns`;
// drain_after_timeout then flags PA_STATUS_TIMEOUT and waits (bounded) for the
// 256-byte copy in flight on stage 1, which the warp writes to `dst` before it
// returns. Nothing traps and nothing is left in flight.
__global__ void __launch_bounds__(32) wait_timeout_selftest_kernel(const uint4* src, uint4* dst,
                                                                   unsigned long long limit_ns,
                                                                   unsigned* status) {
  __shared__ __align__(128) uint4 buf[2][16];   // stage 0 stays empty
  __shared__ __align__(8) uint64_t bars[2];
  const int lane = threadIdx.x;
  const uint32_t bar0 = smem_u32(&bars[0]);
  if (lane == 0) {
    mbar_init(bar0, 2);        // the second arrival never comes
    mbar_init(bar0 + 8, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  if (lane == 0) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar0) : "memory");
    mbar_expect_tx(bar0 + 8, 256);
    bulk_load(smem_u32(&buf[1][0]), src, 256, bar0 + 8);
  }
  __syncwarp();
  if (!mbar_wait(bar0, 0, limit_ns))
    drain_after_timeout<2>(status, bar0, 0, 0u, 1, limit_ns);
  else   // cannot happen (one arrival of two); still, leave no copy in flight
    mbar_wait(bar0 + 8, 0, limit_ns);
  __syncwarp();
  if (lane < 16) dst[lane] = buf[1][lane];
}

// ----------------------------------------------------------------------------
// Host side
// ----------------------------------------------------------------------------
struct DeviceInfo {
  int sms = 0;
};

static std::mutex g_mu;
static DeviceInfo g_dev[64];

static int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  return dev;
}

static int sm_count(int dev) {
  if (dev < 0 || dev >= 64) return 0;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_dev[dev].sms == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    g_dev[dev].sms = v;
  }
  return g_dev[dev].sms;
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

static int gcd_int(int a, int b) {
  while (b) {
    const int t = a % b;
    a = b;
    b = t;
  }
  return a;
}

#endif  // PA_HOST_PART

// Kernel variants: tile tokens, worker warps per CTA, ring depth per warp.
struct Variant {
  int tile, nw, ns;
};
static const Variant kVariants[] = {
    {32, 4, 3},   // 1 (head_dim 128)
    {16, 8, 3},   // 2 (head_dim 128, dup layout only: 9 KB stages)
    {32, 6, 2},   // 3 (head_dim 64 or 128)
    {16, 12, 2},  // 4 (head_dim 128, dup layout only)
    {16, 8, 2},   // 5 (head_dim 64 or 128)
    {16, 4, 2},   // 6 (head_dim 256: 16 KB K+V tiles)
    {16, 5, 2},   // 7 (head_dim 256)
    {64, 6, 2},   // 8 (head_dim 64: 16 KB K+V tiles)
    {32, 3, 2},   // 9 (head_dim 256: 32 KB K+V tiles)
    {32, 4, 2},   // 10 (head_dim 128: 128 KB of tiles in flight per SM)
};
constexpr int kNumVariants = sizeof(kVariants) / sizeof(kVariants[0]);
// Opt-in shared memory per CTA is 227 KB (232448 B), static plus dynamic; the
// kernel's static shared memory (a few words) gets a 1 KB margin.
constexpr int kMaxSmem = 232448 - 1024;

struct Plan {
  int ns = 0;        // 0: balanced
  int grid = 0;
  int W = 0;
  int G = 1, QC = 1;
  int D = 128;       // head_dim
  bool dup = true;
  int variant = 1;   // 1-based index into kVariants
  bool use_cum = false;
  bool wslot_global = false;   // balanced: warps' merge rows in the workspace
  bool long_pieces = false;    // balanced: single-warp groups over long segments
  int slot_cols = 1;
  int gsz = 1;             // balanced: warps per merge group
  int smem = 0;            // dynamic shared memory of the launch
  size_t ws_bytes = 0;
  size_t counters = 0;
  bool generic = false;    // the CUDA-core split + reduce path (uncommon shapes)
  int clu = 0;             // balanced, same length: CTAs per thread-block cluster (0: none)
  int clu_off = 0;         // cluster mode: shared-memory offset of the CTA's piece rows
};

// Shapes the TMA tile kernels do not cover: head_dim 32, or pages that are not
// a multiple of 8 tokens.
static bool generic_shape(const pa_decode_params* p) {
  return p->head_dim == 32 || p->block_size % 8 != 0;
}

#if PA_HOST_PART
// Shared memory a variant needs before the group merge area.
template <bool kDup, int TILE, int NW, int NS, int D>
static int smem_base() {
  return Cfg<kDup, TILE, NW, NS, D>::kSmemBase;
}

// Whether (head_dim, variant, layout) is instantiated.
static bool variant_built(int D, int variant, bool dup) {
  switch (D) {
    case 64: return variant == 3 || variant == 5 || variant == 8;
    case 128:
      return (variant >= 1 && variant <= 5 && (dup || (variant != 2 && variant != 4))) ||
             variant == 10;
    case 256: return variant == 6 || variant == 7 || variant == 9;
    default: return false;
  }
}

static int variant_smem_base(int variant, bool dup, int D) {
  if (D == 64) {
    if (variant == 3) return dup ? smem_base<true, 32, 6, 2, 64>() : smem_base<false, 32, 6, 2, 64>();
    if (variant == 8) return dup ? smem_base<true, 64, 6, 2, 64>() : smem_base<false, 64, 6, 2, 64>();
    return dup ? smem_base<true, 16, 8, 2, 64>() : smem_base<false, 16, 8, 2, 64>();
  }
  if (D == 256) {
    if (variant == 7) return dup ? smem_base<true, 16, 5, 2, 256>() : smem_base<false, 16, 5, 2, 256>();
    if (variant == 9) return dup ? smem_base<true, 32, 3, 2, 256>() : smem_base<false, 32, 3, 2, 256>();
    return dup ? smem_base<true, 16, 4, 2, 256>() : smem_base<false, 16, 4, 2, 256>();
  }
  switch (variant) {
    case 2: return dup ? smem_base<true, 16, 8, 3, 128>() : 0;
    case 3: return dup ? smem_base<true, 32, 6, 2, 128>() : smem_base<false, 32, 6, 2, 128>();
    case 4: return dup ? smem_base<true, 16, 12, 2, 128>() : 0;
    case 5: return dup ? smem_base<true, 16, 8, 2, 128>() : smem_base<false, 16, 8, 2, 128>();
    case 10: return dup ? smem_base<true, 32, 4, 2, 128>() : smem_base<false, 32, 4, 2, 128>();
    default: return dup ? smem_base<true, 32, 4, 3, 128>() : smem_base<false, 32, 4, 3, 128>();
  }
}

static pa_status_t validate(const pa_decode_params* p) {
  if (!p) return PA_ERR_ARG;
  if (p->batch < 0 || p->num_heads <= 0 || p->num_kv_heads <= 0 || p->block_size <= 0 ||
      p->num_blocks <= 0 || p->max_blocks < 0)
    return PA_ERR_ARG;
  if (p->num_heads % p->num_kv_heads != 0) return PA_ERR_ARG;
  if (p->dtype != PA_F16 && p->dtype != PA_BF16) return PA_ERR_ARG;
  if (p->num_splits < 0) return PA_ERR_ARG;
  if (!(p->scale > 0.f) || p->scale > 1e30f) return PA_ERR_ARG;
  if (p->seq_lens == nullptr && p->seq_len < 0) return PA_ERR_ARG;
  if (p->seq_lens == nullptr && static_cast<long long>(p->seq_len) >
                                    static_cast<long long>(p->max_blocks) * p->block_size)
    return PA_ERR_ARG;
  if (p->kernel_variant < 0 || p->kernel_variant > kNumVariants) return PA_ERR_ARG;
  if (p->head_dim != 32 && p->head_dim != 64 && p->head_dim != 128 && p->head_dim != 256)
    return PA_ERR_UNSUPPORTED;
  if (p->block_size > (1 << 20)) return PA_ERR_UNSUPPORTED;
  if (generic_shape(p)) return p->kernel_variant == 0 ? PA_OK : PA_ERR_UNSUPPORTED;
  if (p->kernel_variant != 0) {   // an explicit variant must be built for this head_dim
    const int g = p->num_heads / p->num_kv_heads;
    const bool dup = (g == 1 || g == 2 || g == 4);
    int v = p->kernel_variant;
    if (p->head_dim == 128 && !dup && (v == 2 || v == 4)) v = 5;
    if (!variant_built(p->head_dim, v, dup)) return PA_ERR_UNSUPPORTED;
  }
  return PA_OK;
}

// Everything pa_decode checks before it plans: the parameters, then the
// pointers, alignments and strides of a launch.
static bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; }

static pa_status_t validate_launch(const pa_decode_params* p) {
  const pa_status_t v = validate(p);
  if (v != PA_OK) return v;
  if (!p->q || !p->k_cache || !p->v_cache || !p->block_table || !p->out) return PA_ERR_ARG;
  if (!aligned16(p->q) || !aligned16(p->k_cache) || !aligned16(p->v_cache) || !aligned16(p->out))
    return PA_ERR_ARG;
  if ((p->q_stride_h % 8) || (p->q_stride_b % 8) || (p->out_stride_h % 8) || (p->out_stride_b % 8))
    return PA_ERR_ARG;
  if ((p->k_stride_block % 8) || (p->k_stride_slot % 8) || (p->k_stride_head % 8) ||
      (p->v_stride_block % 8) || (p->v_stride_slot % 8) || (p->v_stride_head % 8))
    return PA_ERR_ARG;
  return PA_OK;
}

// Automatic choice, from B200 sweeps. head_dim 128 (the five benchmark
// shapes): MHA at every page size, and groups larger than 4 query heads,
// stream best as 16-token tiles on 8 warps (B1 S4096 page 128: 24.5 -> 22.6 us
// with L2 flushed; B4 S8192 page 64: 94.6 -> 89.2 us); 2- or 4-head groups as
// 32-token tiles on 6 warps. head_dim 64 (128-byte rows):
// MHA as 32-token tiles on 6 warps, query-head groups as 64-token tiles on 6
// warps. head_dim 256: MHA and pairs as 16-token tiles on 5 warps, groups of
// 4 as 16-token tiles on 4 warps, wider groups as 32-token tiles on 3 warps.
static int pick_variant(const pa_decode_params* p, bool dup, int sms) {
  int v = p->kernel_variant;
  if (v == 0) {
    const int g = p->num_heads / p->num_kv_heads;
    if (p->head_dim == 256)
      // MHA and pairs: 16-token tiles on 5 warps; groups of 4: 16-token tiles
      // on 4 warps, whose merge rows for 4 columns fit in shared memory (B32
      // S1024 Hq32/Hkv8: 57.7 us against 60.1 on 32x3x2); wider groups:
      // 32-token tiles on 3 warps
      v = (g == 1 || g == 2) ? 7 : (g == 4 ? 6 : 9);
    else if (p->head_dim == 64)
      v = g == 1 ? 3 : 8;   // MHA: 32-token tiles on 6 warps; groups: 64-token tiles
    else
      v = (!dup || g == 1) ? 5 : 3;
    // Query-head groups whose segments can exceed 8 tiles of 32 tokens. 32x6x2
    // keeps its warps' merge rows in shared memory only up to 2 query columns.
    // With more columns: no more segments than SMs -> 32x6x2 as single-warp
    // groups whose pieces meet in the merge pass (B1 S4096 Hq32/Hkv8 15.4 us
    // against 19.5 on 16x8x2, B16 S1024 25.6 against 27.8, B1 S32768
    // Hq32/Hkv4 25.8 against 27.8), except same-length rows of >= 8192 tokens
    // that the cluster schedule covers on 16x8x2 (B8 S32768: 170.7 against
    // 174.7); more segments than SMs -> 16x8x2, whose merge rows fit (B64 S512:
    // 37.0 against 40.3 with 32x6x2's rows in the workspace).
    if (p->head_dim == 128 && g > 1) {
      const long long cap = static_cast<long long>(p->max_blocks) * p->block_size;
      const long long nseg = static_cast<long long>(p->batch) * p->num_kv_heads * ((g + 7) / 8);
      const int cols = std::min(g, 8);
      const bool fits = variant_smem_base(3, dup, 128) + 6 * 2 * (128 + 4) * 4 * cols <= kMaxSmem;
      if (!fits && (cap + 31) / 32 > 8) {
        const long long clu = nseg > 0 ? std::min<long long>(8, sms / nseg) : 0;
        const bool clusters = p->seq_lens == nullptr && p->seq_len >= 8192 && clu >= 2 &&
                              4 * nseg * clu >= 3ll * sms;
        v = (nseg <= sms && !clusters) ? 3 : 5;
      }
      // 16x8x2 without duplicated columns holds the merge rows of at most 7
      // query columns; with 8 and more segments than SMs they would go to the
      // workspace, so 32x4x2, whose rows fit, takes over (the C5 shards of 8
      // ranks, B256 Hq8/Hkv1: 187.5 -> 155.9 us; of 4 ranks 316 -> 287;
      // B128 S<=1024 Hq64/Hkv8 79.8 -> 61.5 us flushed).
      if (v == 5 && !dup && nseg > sms && (cap + 15) / 16 > 8 &&
          variant_smem_base(5, false, 128) + 8 * 2 * (128 + 4) * 4 * cols > kMaxSmem)
        v = 10;
    }
  }
  if (p->head_dim == 128 && !dup && (v == 2 || v == 4)) v = 5;
  return variant_built(p->head_dim, v, dup) ? v : 0;   // 0: not built for this head_dim
}

// Bytes of the balanced schedule's group partials (rows, then LSEs), rounded
// to 16 bytes so that what follows stays aligned.
static size_t group_slot_bytes(const Plan& pl, size_t slots) {
  const size_t b = slots * pl.slot_cols * (pl.D + 1) * sizeof(float);
  return (b + 15) & ~size_t(15);
}

// Cluster mode (same-length rows, whole-CTA groups whose merge rows are in
// shared memory, segments longer than a CTA's share): one cluster of `clu`
// CTAs per segment, clu = min(8, sms / segments) >= 2, used when the clusters
// still cover >= 3/4 of the SMs. The CTAs' pieces meet in distributed shared
// memory at the end of the kernel instead of through L2 arrivals and a merge
// by the last CTA (B1 H32 S4096, page 128: the cross-CTA tail of ~3.5 us).
// Cluster launches the device could not hold at once (cudaOccupancyMaxActiveClusters),
// so that later calls plan without clusters directly.
struct CluBad { int dev, variant, D, dup, dtype, clu, smem; };
static CluBad g_clu_bad[32];
static int g_nclu_bad = 0;

static bool cluster_known_bad(const CluBad& k) {
  std::lock_guard<std::mutex> lk(g_mu);
  for (int i = 0; i < g_nclu_bad; ++i) {
    const CluBad& e = g_clu_bad[i];
    if (e.dev == k.dev && e.variant == k.variant && e.D == k.D && e.dup == k.dup &&
        e.dtype == k.dtype && e.clu == k.clu && e.smem == k.smem)
      return true;
  }
  return false;
}

static void cluster_mark_bad(const CluBad& k) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_nclu_bad < 32) g_clu_bad[g_nclu_bad++] = k;
}

static CluBad cluster_key(const pa_decode_params* p, const Plan& pl) {
  return CluBad{current_device(), pl.variant, pl.D, pl.dup ? 1 : 0, p->dtype, pl.clu, pl.smem};
}

static void plan_cluster(const pa_decode_params* p, int sms, Plan& pl) {
  if (pl.ns != 0 || pl.use_cum || pl.gsz == 1 || pl.wslot_global || p->seq_len <= 0) return;
  const Variant& v = kVariants[pl.variant - 1];
  const long long nseg = static_cast<long long>(p->batch) * p->num_kv_heads * pl.QC;
  const long long nt = (p->seq_len + v.tile - 1) / v.tile;
  if (nseg < 1 || 2 * nseg > sms) return;
  const int clu = static_cast<int>(std::min<long long>(8, sms / nseg));
  if (clu < 2 || 4 * nseg * clu < 3ll * sms) return;
  // only where the plain schedule splits segments between CTAs
  const long long groups = pl.W / pl.gsz;
  if (std::max<long long>((nseg * nt + groups - 1) / groups, pl.gsz) >= nt) return;
  const long long per = (nt + clu - 1) / clu;   // units per CTA
  if ((clu - 1) * per >= nt) return;            // every rank has units
  const long long off = (static_cast<long long>(pl.smem) - 1024 + 15) & ~15ll;
  // rank 0's arrival barrier (16 B), then every CTA's piece rows
  const long long bytes = 16 + static_cast<long long>(clu) * pl.slot_cols * (pl.D + 4) * 4;
  if (off + bytes + 1024 > kMaxSmem) return;
  Plan c = pl;
  c.clu = clu;
  c.clu_off = static_cast<int>(off);
  c.smem = static_cast<int>(off + bytes + 1024);
  c.grid = static_cast<int>(nseg) * clu;
  c.W = c.grid * v.nw;
  if (cluster_known_bad(cluster_key(p, c))) return;
  pl = c;
}

static pa_status_t make_plan(const pa_decode_params* p, int sms, Plan& pl,
                             bool allow_cluster = true) {
  pl.G = p->num_heads / p->num_kv_heads;
  pl.QC = (pl.G + 7) / 8;
  pl.dup = (pl.G == 1 || pl.G == 2 || pl.G == 4);
  pl.D = p->head_dim;
  if (generic_shape(p)) {
    // One warp per (row, query head, split), four warps per CTA; splits as
    // given, else the reference heuristic (torch_kernel.py:19-25).
    pl.generic = true;
    pl.variant = 0;
    const long long cap = static_cast<long long>(p->max_blocks) * p->block_size;
    pl.ns = p->num_splits > 0
                ? p->num_splits
                : pa_num_splits_heuristic(p->batch, p->num_heads,
                                          static_cast<int>(cap > 0x7fffffff ? 0x7fffffff : cap),
                                          p->block_size, sms);
    const long long workers = static_cast<long long>(p->batch) * p->num_heads * pl.ns;
    if (workers > 0x7fffffffll * 4) return PA_ERR_UNSUPPORTED;
    pl.W = static_cast<int>(std::min<long long>(workers, 0x7fffffffll));
    pl.grid = static_cast<int>((workers + 3) / 4);
    pl.ws_bytes = (p->o_partial && p->lse_partial)
                      ? 0
                      : static_cast<size_t>(workers) * (pl.D + 1) * sizeof(float);
    pl.counters = 0;
    return PA_OK;
  }
  pl.variant = pick_variant(p, pl.dup, sms);
  if (pl.variant == 0) return PA_ERR_UNSUPPORTED;
  const Variant& v = kVariants[pl.variant - 1];
  const long long nseg = static_cast<long long>(p->num_kv_heads) * pl.QC;
  const long long cap = static_cast<long long>(p->max_blocks) * p->block_size;
  pl.ns = p->num_splits;
  if (pl.ns == 0) {
    const long long nt = (cap + v.tile - 1) / v.tile;
    // Unit indices must fit int32; very large batches with per-row lengths
    // use the split schedule with the reference heuristic instead.
    if ((p->seq_lens != nullptr && p->batch > kCumMax) ||
        static_cast<long long>(p->batch) * nseg * nt > 0x7fffffffll) {
      const int s_max = static_cast<int>(cap > 0x7fffffff ? 0x7fffffff : cap);
      pl.ns = pa_num_splits_heuristic(p->batch, p->num_heads, s_max, p->block_size, sms);
    }
  }
  pl.slot_cols = std::min(pl.G, 8);
  if (pl.ns == 0) {
    pl.grid = sms;
    pl.W = pl.grid * v.nw;
    pl.use_cum = p->seq_lens != nullptr;
    // Merge pieces inside a CTA through shared memory when the warps' rows fit.
    const int base = variant_smem_base(pl.variant, pl.dup, pl.D);
    // Groups are whole CTAs whose warps merge through shared memory when their
    // merge rows fit beside the stages. Otherwise: single-warp groups when no
    // segment can exceed 8 tiles (no cross-group merge of more than 8 pieces)
    // or when there are no more segments than CTAs (their pieces merge in the
    // merge pass), else whole CTAs with the warps' merge rows in the workspace
    // (a long segment would otherwise split into one piece per warp, merged by
    // one warp).
    const int group_bytes = v.nw * 2 * (pl.D + 4) * 4 * pl.slot_cols;
    const long long max_nt = (cap + v.tile - 1) / v.tile;
    pl.gsz = v.nw;
    if (base + group_bytes > kMaxSmem) {
      if (max_nt <= 8) {
        pl.gsz = 1;
      } else if (static_cast<long long>(p->batch) * nseg <= pl.grid) {
        // No more segments than CTAs: each spans CTAs, and one warp per CTA
        // would merge its warps' rows column after column from the workspace
        // (an L2 round trip each). Single-warp groups instead, whose pieces
        // all merge in the merge pass after the decode kernel.
        pl.gsz = 1;
        pl.long_pieces = true;
      } else {
        pl.wslot_global = true;
      }
    }
    pl.smem = base + ((pl.gsz > 1 && !pl.wslot_global) ? group_bytes : 0);
    const size_t slots = static_cast<size_t>(2) * (pl.W / pl.gsz);   // two per group
    pl.ws_bytes = group_slot_bytes(pl, slots);
    if (pl.wslot_global) pl.ws_bytes += static_cast<size_t>(pl.grid) * group_bytes;
  } else {
    pl.smem = variant_smem_base(pl.variant, pl.dup, pl.D);
    const long long workers = static_cast<long long>(p->batch) * nseg * pl.ns;
    if (workers > 0x7fffffffll) return PA_ERR_UNSUPPORTED;
    pl.W = static_cast<int>(workers);
    pl.grid = static_cast<int>((workers + v.nw - 1) / v.nw);
    const size_t rows = static_cast<size_t>(p->batch) * p->num_heads * pl.ns;
    pl.ws_bytes = (p->o_partial && p->lse_partial) ? 0 : rows * (pl.D + 1) * sizeof(float);
  }
  pl.counters = static_cast<size_t>(p->batch) * nseg;
  if (allow_cluster) plan_cluster(p, sms, pl);
  return PA_OK;
}

// Tensor map of one paged cache [num_blocks, block_size, Hkv, D], with the
// dimensions ordered (64 dims, slot, 64-dim chunk, head, block) so that one
// box of {64, R, D/64, 1, 1} lands as [chunk][R rows][128 B]: all chunks of R
// token rows in one copy. The strides are the caller's (multiples of 16 bytes).
static bool encode_cache_map(CUtensorMap* map, const pa_decode_params* p, const void* base,
                             int64_t s_block, int64_t s_slot, int64_t s_head, int rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  const CUtensorMapDataType dt =
      p->dtype == PA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[5] = {64, static_cast<cuuint64_t>(p->block_size),
                        static_cast<cuuint64_t>(p->head_dim / 64),
                        static_cast<cuuint64_t>(p->num_kv_heads),
                        static_cast<cuuint64_t>(p->num_blocks)};
  cuuint64_t strides[4] = {static_cast<cuuint64_t>(s_slot) * 2, 128,
                           static_cast<cuuint64_t>(s_head) * 2,
                           static_cast<cuuint64_t>(s_block) * 2};
  cuuint32_t box[5] = {64, static_cast<cuuint32_t>(rows),
                       static_cast<cuuint32_t>(p->head_dim / 64), 1, 1};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  // L2 fills widened to 256 B suit rows of >= 256 B; a 128-byte row (D = 64)
  // would drag its neighbouring head's row along.
  const CUtensorMapL2promotion promo = p->head_dim == 64 ? CU_TENSOR_MAP_L2_PROMOTION_L2_128B
                                                         : CU_TENSOR_MAP_L2_PROMOTION_L2_256B;
  const CUresult r = fn(map, dt, 5, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, promo,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Encoded tensor maps are reused across calls: a decode loop passes the same
// K/V cache pointers every step. Small round-robin cache, keyed by everything
// the encoding depends on.
struct MapKey {
  int dev, dtype, rows, head_dim;
  const void* base;
  int64_t dims[3];      // block_size, num_kv_heads, num_blocks
  int64_t strides[3];   // block, slot, head (elements)
  bool operator==(const MapKey& o) const {
    return dev == o.dev && dtype == o.dtype && rows == o.rows && head_dim == o.head_dim &&
           base == o.base && memcmp(dims, o.dims, sizeof(dims)) == 0 &&
           memcmp(strides, o.strides, sizeof(strides)) == 0;
  }
};
constexpr int kMapCache = 16;
static MapKey g_map_keys[kMapCache];
static CUtensorMap g_maps[kMapCache];
static bool g_map_valid[kMapCache];
static int g_map_next = 0;

static bool cached_cache_map(CUtensorMap* map, const pa_decode_params* p, int dev, const void* base,
                             int64_t s_block, int64_t s_slot, int64_t s_head, int rows) {
  MapKey key;
  memset(&key, 0, sizeof(key));
  key.dev = dev;
  key.dtype = p->dtype;
  key.rows = rows;
  key.head_dim = p->head_dim;
  key.base = base;
  key.dims[0] = p->block_size;
  key.dims[1] = p->num_kv_heads;
  key.dims[2] = p->num_blocks;
  key.strides[0] = s_block;
  key.strides[1] = s_slot;
  key.strides[2] = s_head;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    for (int i = 0; i < kMapCache; ++i)
      if (g_map_valid[i] && g_map_keys[i] == key) {
        *map = g_maps[i];
        return true;
      }
  }
  if (!encode_cache_map(map, p, base, s_block, s_slot, s_head, rows)) return false;
  std::lock_guard<std::mutex> lk(g_mu);
  const int i = g_map_next;
  g_map_next = (g_map_next + 1) % kMapCache;
  g_map_keys[i] = key;
  g_maps[i] = *map;
  g_map_valid[i] = true;
  return true;
}

#endif  // PA_HOST_PART

template <typename T, bool kDup, int TILE, int NW, int NS, int D, bool kSplit, bool kCum,
          bool kClu>
cudaError_t launch_kernel(const Plan& pl, const CUtensorMap& mk, const CUtensorMap& mv,
                          const KParams& kp, cudaStream_t stream, int dev) {
  using C = Cfg<kDup, TILE, NW, NS, D>;
  static_assert(C::kSmemBase <= kMaxSmem, "shared memory plan exceeds 227 KB");
  static std::mutex mu;
  static bool attr_set[64] = {false};
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!attr_set[dev]) {
      const cudaError_t e = cudaFuncSetAttribute(pa_decode_kernel<T, kDup, TILE, NW, NS, D, kSplit, kCum, kClu>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 kMaxSmem);
      if (e != cudaSuccess) return e;
      attr_set[dev] = true;
    }
  }
  // Programmatic stream serialisation: the grid may be scheduled while the
  // previous kernel in the stream finishes; the kernel's griddepcontrol.wait
  // orders all of its memory accesses after that kernel.
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(NW * 32);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (kClu) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = pl.clu;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
    // Every cluster must be resident at once (one CTA per SM): checked once
    // per device, cluster size and shared-memory size.
    struct Seen { int dev, clu, smem, ok; };
    static Seen seen[16];
    static int nseen = 0;
    int ok = -1;
    {
      std::lock_guard<std::mutex> lk(mu);
      for (int i = 0; i < nseen; ++i)
        if (seen[i].dev == dev && seen[i].clu == pl.clu && seen[i].smem == pl.smem) ok = seen[i].ok;
    }
    if (ok < 0) {
      int n = 0;
      const cudaError_t q = cudaOccupancyMaxActiveClusters(
          &n, pa_decode_kernel<T, kDup, TILE, NW, NS, D, kSplit, kCum, kClu>, &cfg);
      ok = (q == cudaSuccess && n * pl.clu >= pl.grid) ? 1 : 0;
      if (q != cudaSuccess) (void)cudaGetLastError();
      std::lock_guard<std::mutex> lk(mu);
      if (nseen < 16) seen[nseen++] = Seen{dev, pl.clu, pl.smem, ok};
    }
    if (!ok) return cudaErrorCooperativeLaunchTooLarge;   // the caller re-plans without clusters
  }
  return cudaLaunchKernelEx(&cfg, pa_decode_kernel<T, kDup, TILE, NW, NS, D, kSplit, kCum, kClu>, mk, mv, kp);
}

// Every decode kernel the dispatch below can launch, as (variant, layout) per
// head_dim and dtype; PFX is `extern` for declarations, empty for definitions.
#define PA_LK(T, DUP, TILE, NW, NS, D, SPLIT, CUM, CLU)                                     \
  cudaError_t launch_kernel<T, DUP, TILE, NW, NS, D, SPLIT, CUM, CLU>(                      \
      const Plan&, const CUtensorMap&, const CUtensorMap&, const KParams&, cudaStream_t, int)
#define PA_BOTH(PFX, T, DUP, TILE, NW, NS, D)                        \
  PFX template PA_LK(T, DUP, TILE, NW, NS, D, false, false, false);  \
  PFX template PA_LK(T, DUP, TILE, NW, NS, D, false, false, true);   \
  PFX template PA_LK(T, DUP, TILE, NW, NS, D, false, true, false);   \
  PFX template PA_LK(T, DUP, TILE, NW, NS, D, true, false, false);
#define PA_D128(PFX, T)                                                              \
  PA_BOTH(PFX, T, true, 32, 4, 3, 128) PA_BOTH(PFX, T, false, 32, 4, 3, 128)         \
  PA_BOTH(PFX, T, true, 16, 8, 3, 128)                                               \
  PA_BOTH(PFX, T, true, 32, 6, 2, 128) PA_BOTH(PFX, T, false, 32, 6, 2, 128)         \
  PA_BOTH(PFX, T, true, 16, 12, 2, 128)                                              \
  PA_BOTH(PFX, T, true, 16, 8, 2, 128) PA_BOTH(PFX, T, false, 16, 8, 2, 128)         \
  PA_BOTH(PFX, T, true, 32, 4, 2, 128) PA_BOTH(PFX, T, false, 32, 4, 2, 128)
#define PA_D64(PFX, T)                                                               \
  PA_BOTH(PFX, T, true, 32, 6, 2, 64) PA_BOTH(PFX, T, false, 32, 6, 2, 64)           \
  PA_BOTH(PFX, T, true, 16, 8, 2, 64) PA_BOTH(PFX, T, false, 16, 8, 2, 64)           \
  PA_BOTH(PFX, T, true, 64, 6, 2, 64) PA_BOTH(PFX, T, false, 64, 6, 2, 64)
#define PA_D256(PFX, T)                                                              \
  PA_BOTH(PFX, T, true, 16, 4, 2, 256) PA_BOTH(PFX, T, false, 16, 4, 2, 256)         \
  PA_BOTH(PFX, T, true, 16, 5, 2, 256) PA_BOTH(PFX, T, false, 16, 5, 2, 256)         \
  PA_BOTH(PFX, T, true, 32, 3, 2, 256) PA_BOTH(PFX, T, false, 32, 3, 2, 256)

#if PA_HOST_PART
#if defined(PA_PART)
// Parts 1-4 hold the definitions.
PA_D128(extern, __half)
PA_D128(extern, __nv_bfloat16)
PA_D64(extern, __half)
PA_D64(extern, __nv_bfloat16)
PA_D256(extern, __half)
PA_D256(extern, __nv_bfloat16)
#endif

// The split schedule, the balanced schedule over same-length rows (plain, or
// as thread-block clusters) and the balanced schedule over per-row lengths are
// separate kernels: none carries another's code (short steps are bound by
// instruction fetch).
template <typename T, bool kDup, int TILE, int NW, int NS, int D>
static cudaError_t launch_one(const Plan& pl, const CUtensorMap& mk, const CUtensorMap& mv,
                              const KParams& kp, cudaStream_t stream, int dev) {
  if (pl.ns != 0)
    return launch_kernel<T, kDup, TILE, NW, NS, D, true, false, false>(pl, mk, mv, kp, stream, dev);
  if (pl.use_cum)
    return launch_kernel<T, kDup, TILE, NW, NS, D, false, true, false>(pl, mk, mv, kp, stream, dev);
  if (pl.clu)
    return launch_kernel<T, kDup, TILE, NW, NS, D, false, false, true>(pl, mk, mv, kp, stream, dev);
  return launch_kernel<T, kDup, TILE, NW, NS, D, false, false, false>(pl, mk, mv, kp, stream, dev);
}

template <typename T, bool kDup>
static cudaError_t launch(const Plan& pl, const CUtensorMap& mk, const CUtensorMap& mv,
                          const KParams& kp, cudaStream_t stream, int dev) {
  if (pl.D == 64) {
    if (pl.variant == 3) return launch_one<T, kDup, 32, 6, 2, 64>(pl, mk, mv, kp, stream, dev);
    if (pl.variant == 8) return launch_one<T, kDup, 64, 6, 2, 64>(pl, mk, mv, kp, stream, dev);
    return launch_one<T, kDup, 16, 8, 2, 64>(pl, mk, mv, kp, stream, dev);
  }
  if (pl.D == 256) {
    if (pl.variant == 7) return launch_one<T, kDup, 16, 5, 2, 256>(pl, mk, mv, kp, stream, dev);
    if (pl.variant == 9) return launch_one<T, kDup, 32, 3, 2, 256>(pl, mk, mv, kp, stream, dev);
    return launch_one<T, kDup, 16, 4, 2, 256>(pl, mk, mv, kp, stream, dev);
  }
  switch (pl.variant) {
    case 2:
      if constexpr (kDup) return launch_one<T, kDup, 16, 8, 3, 128>(pl, mk, mv, kp, stream, dev);
      break;
    case 3:
      return launch_one<T, kDup, 32, 6, 2, 128>(pl, mk, mv, kp, stream, dev);
    case 4:
      if constexpr (kDup) return launch_one<T, kDup, 16, 12, 2, 128>(pl, mk, mv, kp, stream, dev);
      break;
    case 5:
      return launch_one<T, kDup, 16, 8, 2, 128>(pl, mk, mv, kp, stream, dev);
    case 10:
      return launch_one<T, kDup, 32, 4, 2, 128>(pl, mk, mv, kp, stream, dev);
    default:
      break;
  }
  return launch_one<T, kDup, 32, 4, 3, 128>(pl, mk, mv, kp, stream, dev);
}

template <typename T, int D, bool kCum>
static cudaError_t launch_merge_kernel(const MergeParams& m, dim3 grid, cudaStream_t stream) {
  // Dependent launch: the grid may be scheduled while the decode kernel runs;
  // griddepcontrol.wait orders its reads after that kernel's completion.
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = grid;
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, merge_segments_kernel<T, D, kCum>, m);
}

template <typename T>
static cudaError_t launch_merge(const MergeParams& m, int D, bool cum, dim3 grid,
                                cudaStream_t stream) {
  if (D == 64)
    return cum ? launch_merge_kernel<T, 64, true>(m, grid, stream)
               : launch_merge_kernel<T, 64, false>(m, grid, stream);
  if (D == 256)
    return cum ? launch_merge_kernel<T, 256, true>(m, grid, stream)
               : launch_merge_kernel<T, 256, false>(m, grid, stream);
  return cum ? launch_merge_kernel<T, 128, true>(m, grid, stream)
             : launch_merge_kernel<T, 128, false>(m, grid, stream);
}

// The CUDA-core path: the split kernel, then the reduce kernel, on `stream`.
static cudaError_t launch_generic(const pa_decode_params* p, const Plan& pl,
                                  cudaStream_t stream) {
  GenParams g;
  memset(&g, 0, sizeof(g));
  g.q = static_cast<const char*>(p->q);
  g.q_sb = p->q_stride_b * 2;
  g.q_sh = p->q_stride_h * 2;
  g.kc = static_cast<const char*>(p->k_cache);
  g.vc = static_cast<const char*>(p->v_cache);
  g.k_sb = p->k_stride_block * 2;
  g.k_ss = p->k_stride_slot * 2;
  g.k_sh = p->k_stride_head * 2;
  g.v_sb = p->v_stride_block * 2;
  g.v_ss = p->v_stride_slot * 2;
  g.v_sh = p->v_stride_head * 2;
  g.bt = p->block_table;
  g.bt_sb = p->bt_stride_b;
  g.max_blocks = p->max_blocks;
  g.seq_lens = p->seq_lens;
  g.seq_len = p->seq_lens ? 0 : p->seq_len;
  g.B = p->batch;
  g.Hq = p->num_heads;
  g.G = pl.G;
  g.bs = p->block_size;
  g.NB = p->num_blocks;
  g.ns = pl.ns;
  g.scale_log2 = p->scale * kLog2e;
  if (p->o_partial && p->lse_partial) {
    g.o_part = p->o_partial;
    g.lse_part = p->lse_partial;
  } else {
    const size_t rows = static_cast<size_t>(p->batch) * p->num_heads * pl.ns;
    g.o_part = static_cast<float*>(p->workspace);
    g.lse_part = g.o_part + rows * pl.D;
  }
  g.out = static_cast<char*>(p->out);
  g.o_sb = p->out_stride_b * 2;
  g.o_sh = p->out_stride_h * 2;
  g.lse = p->lse;
  g.status = p->status;
  const long long rows_hq = static_cast<long long>(p->batch) * p->num_heads;
  const dim3 grid_split(pl.grid), grid_reduce(static_cast<unsigned>((rows_hq + 3) / 4));
  const bool bf = p->dtype == PA_BF16;
#define PA_GENERIC(DIM)                                                                  \
  if (pl.D == DIM) {                                                                     \
    if (bf) {                                                                            \
      generic_split_kernel<__nv_bfloat16, DIM><<<grid_split, 128, 0, stream>>>(g);       \
      generic_reduce_kernel<__nv_bfloat16, DIM><<<grid_reduce, 128, 0, stream>>>(g);     \
    } else {                                                                             \
      generic_split_kernel<__half, DIM><<<grid_split, 128, 0, stream>>>(g);              \
      generic_reduce_kernel<__half, DIM><<<grid_reduce, 128, 0, stream>>>(g);            \
    }                                                                                    \
    return cudaGetLastError();                                                           \
  }
  PA_GENERIC(32)
  PA_GENERIC(64)
  PA_GENERIC(128)
  PA_GENERIC(256)
#undef PA_GENERIC
  return cudaErrorInvalidValue;
}

// Kernel parameters of one call (the plan's schedule constants, the
// workspace carve-up and the multiply-shift divisors).
static void build_kparams(const pa_decode_params* p, const Plan& pl, KParams& kp) {
  memset(&kp, 0, sizeof(kp));
  kp.q = static_cast<const char*>(p->q);
  kp.q_sb = p->q_stride_b * 2;
  kp.q_sh = p->q_stride_h * 2;
  kp.out = static_cast<char*>(p->out);
  kp.o_sb = p->out_stride_b * 2;
  kp.o_sh = p->out_stride_h * 2;
  kp.lse = p->lse;
  kp.bt = p->block_table;
  kp.bt_sb = p->bt_stride_b;
  kp.max_blocks = p->max_blocks;
  kp.seq_lens = p->seq_lens;
  kp.seq_len = p->seq_lens ? 0 : p->seq_len;
  kp.B = p->batch;
  kp.Hq = p->num_heads;
  kp.Hkv = p->num_kv_heads;
  kp.G = pl.G;
  kp.QC = pl.QC;
  kp.bs = p->block_size;
  kp.NB = p->num_blocks;
  kp.ns = pl.ns;
  kp.scale_log2 = p->scale * kLog2e;
  if (pl.ns == 0) {
    float* ws = static_cast<float*>(p->workspace);
    const size_t slots = static_cast<size_t>(2) * (pl.W / pl.gsz);
    kp.o_part = ws;
    kp.lse_part = ws + slots * pl.slot_cols * pl.D;
    if (pl.wslot_global)
      kp.wslots = ws + group_slot_bytes(pl, slots) / sizeof(float);
  } else if (p->o_partial && p->lse_partial) {
    kp.o_part = p->o_partial;
    kp.lse_part = p->lse_partial;
  } else {
    float* ws = static_cast<float*>(p->workspace);
    const size_t rows = static_cast<size_t>(p->batch) * p->num_heads * pl.ns;
    kp.o_part = ws;
    kp.lse_part = ws + rows * pl.D;
  }
  kp.counters = p->counters;
  kp.status = p->status;
  const int tile = kVariants[pl.variant - 1].tile;
  kp.R = gcd_int(p->block_size, tile);
  kp.lspt = 0;
  while ((kp.R << kp.lspt) < tile) ++kp.lspt;
  kp.lR = 0;
  while ((1 << kp.lR) < kp.R) ++kp.lR;
  kp.bs_log2 = -1;
  for (int k = 0; k < 31; ++k)
    if ((1 << k) == p->block_size) kp.bs_log2 = k;
  kp.W = pl.W;
  kp.slot_cols = pl.slot_cols;
  kp.gsz = pl.gsz;
  kp.zero_rows = (p->seq_lens != nullptr || p->seq_len == 0) ? 1 : 0;
  if (pl.ns == 0) {
    const int ngroups = pl.W / pl.gsz;
    kp.nt_u = p->seq_lens ? 0 : (p->seq_len + tile - 1) / tile;
    kp.per_row = p->num_kv_heads * pl.QC * kp.nt_u;
    kp.U = p->batch * kp.per_row;            // fits int32: checked by make_plan
    kp.P = std::max((kp.U + ngroups - 1) / ngroups, pl.gsz);
    // Whole segments per group when that costs at most 25 % more units in the
    // fullest group (40 % with query-head groups, whose split segments would
    // otherwise go through the merge pass): no segment then crosses a group,
    // so no piece needs a cross-CTA merge, whose round trips land on the tail
    // of the step. Same-length steps, L2 flushed: B32 S1024 MHA at D = 256
    // (+16 %, 128 CTAs) 91.4 -> 86.4 us, B12 S1024 H32 41.5 -> 39.1, B40 S1024
    // Hq32/Hkv8 (+39 %) 43.5 -> 39.2; B10 S2048 H32 (+39 %) 60.6 -> 61.9 and
    // B5 S4096 H32 (+85 %, 80 CTAs) 61.6 -> 78.1 stay unaligned.
    const long long nseg_total = static_cast<long long>(p->batch) * p->num_kv_heads * pl.QC;
    if (kp.nt_u > 0 && nseg_total >= ngroups) {
      const long long aligned = (nseg_total + ngroups - 1) / ngroups * kp.nt_u;
      const long long limit = pl.slot_cols > 1 ? 140 : 125;
      if (aligned * 100 <= static_cast<long long>(kp.P) * limit && aligned >= pl.gsz)
        kp.P = static_cast<int>(aligned);
    }
    kp.Pw = (kp.P + pl.gsz - 1) / pl.gsz;
    kp.div_row = make_fastdiv(static_cast<uint32_t>(kp.per_row));
    kp.div_nt = make_fastdiv(static_cast<uint32_t>(kp.nt_u));
    kp.div_ng = make_fastdiv(static_cast<uint32_t>(ngroups));
  }
  kp.div_qc = make_fastdiv(static_cast<uint32_t>(pl.QC));
  kp.div_bs = make_fastdiv(static_cast<uint32_t>(p->block_size));
  const long long cap = static_cast<long long>(p->max_blocks) * p->block_size;
  kp.max_nt = static_cast<int>(std::min<long long>((cap + tile - 1) / tile, 0x3fffffff));
  if (pl.clu) {
    kp.clu = pl.clu;
    kp.clu_off = pl.clu_off;
    kp.P = (kp.nt_u + pl.clu - 1) / pl.clu;
    kp.Pw = (kp.P + pl.gsz - 1) / pl.gsz;
  }
}

// Whether the segments that cross group boundaries merge in
// merge_segments_kernel rather than by the last group's warp inside the
// decode kernel, and that kernel's grid. The pass costs a dependent launch
// (about 5 us on B200); the in-kernel merge costs an L2 round trip per column
// and per 8 pieces on the step's tail, which is exposed when few long segments
// finish together. From B200 sweeps: the pass wins for query-head groups
// (two or more columns) and for single columns over more than 8 pieces, and
// loses for single-warp groups (short segments, merged in parallel by many
// warps) and for per-row lengths with more segments than groups.
// Single-warp groups over long segments (pl.long_pieces) always take the pass.
static bool want_post_merge(const pa_decode_params* p, const Plan& pl, const KParams& kp,
                            dim3& grid, int& by_segment, int& col_split) {
  if (pl.ns != 0 || pl.clu || (pl.gsz == 1 && !pl.long_pieces)) return false;
  const int ngroups = pl.W / pl.gsz;
  if (ngroups < 2) return false;
  const long long nseg_total = static_cast<long long>(p->batch) * p->num_kv_heads * pl.QC;
  long long pieces;   // groups a segment may span
  if (!pl.use_cum) {
    // Segments start at multiples of nt_u: none crosses a group boundary when
    // P is one, or when one group holds every unit.
    if (kp.nt_u == 0 || kp.U <= kp.P || kp.P % kp.nt_u == 0) return false;
    pieces = (kp.nt_u + kp.P - 2) / kp.P + 1;
    if (!pl.long_pieces && pl.slot_cols < 2 && pieces <= 8) return false;
  } else {
    // lengths are on the device: judged by segments per group
    if (!pl.long_pieces && nseg_total * (pl.slot_cols < 2 ? 8 : 1) >= ngroups) return false;
    pieces = ngroups / std::max(1ll, nseg_total) + 1;
  }
  by_segment = nseg_total <= ngroups - 1 ? 1 : 0;
  // More than 32 pieces a column: one column per CTA, its eight warps over the pieces.
  col_split = (pieces > 32 && pl.slot_cols > 1) ? 1 : 0;
  grid = dim3(by_segment ? static_cast<unsigned>(nseg_total) : static_cast<unsigned>(ngroups - 1),
              col_split ? static_cast<unsigned>(pl.slot_cols) : 1u);
  return true;
}

}  // namespace pa

using namespace pa;

extern "C" {

int32_t pa_abi_version(void) { return PA_ABI_VERSION; }

const char* pa_status_string(pa_status_t s) {
  switch (s) {
    case PA_OK: return "ok";
    case PA_ERR_ARG: return "invalid argument";
    case PA_ERR_UNSUPPORTED: return "unsupported configuration";
    case PA_ERR_LAUNCH: return "CUDA launch failure";
    case PA_ERR_WORKSPACE: return "workspace too small";
  }
  return "unknown status";
}

int32_t pa_num_splits_heuristic(int32_t batch, int32_t heads, int32_t seq_len, int32_t block_size,
                                int32_t sm_count) {
  // paged_attention/torch_kernel.py:19-25, with the SM count of the caller's device.
  if (batch <= 0 || heads <= 0 || block_size <= 0) return 1;
  const long long target = 4ll * sm_count;
  const long long by_sm = std::max(1ll, target / (static_cast<long long>(batch) * heads));
  const long long by_len = (static_cast<long long>(seq_len) + block_size - 1) / block_size;
  return static_cast<int32_t>(std::max(1ll, std::min(by_len, by_sm)));
}

int32_t pa_device_sm_count(void) { return sm_count(current_device()); }

pa_status_t pa_decode_workspace(const pa_decode_params* p, size_t* workspace_bytes,
                                size_t* counter_count) {
  const pa_status_t v = validate(p);
  if (v != PA_OK) return v;
  const int sms = sm_count(current_device());
  if (sms <= 0) return PA_ERR_LAUNCH;
  Plan pl;
  const pa_status_t s = make_plan(p, sms, pl);
  if (s != PA_OK) return s;
  if (workspace_bytes) *workspace_bytes = pl.ws_bytes;
  if (counter_count) *counter_count = pl.counters;
  return PA_OK;
}

pa_status_t pa_decode_plan(const pa_decode_params* p, pa_decode_plan_info* info) {
  if (!info) return PA_ERR_ARG;
  const pa_status_t v = validate(p);
  if (v != PA_OK) return v;
  const int sms = sm_count(current_device());
  if (sms <= 0) return PA_ERR_LAUNCH;
  Plan pl;
  const pa_status_t s = make_plan(p, sms, pl);
  if (s != PA_OK) return s;
  memset(info, 0, sizeof(*info));
  if (pl.generic) {
    info->tile_tokens = 32;
    info->warps = 4;
    info->grid = pl.grid;
    info->num_splits = pl.ns;
    info->kernels = p->batch == 0 ? 0 : 2;
    info->generic_path = 1;
    info->workspace_bytes = pl.ws_bytes;
    return PA_OK;
  }
  KParams kp;
  build_kparams(p, pl, kp);
  dim3 merge_grid(1);
  int by_segment = 0, col_split = 0;
  const bool post = p->batch > 0 && want_post_merge(p, pl, kp, merge_grid, by_segment, col_split);
  const Variant& var = kVariants[pl.variant - 1];
  info->kernel_variant = pl.variant;
  info->tile_tokens = var.tile;
  info->warps = var.nw;
  info->stages = var.ns;
  info->grid = pl.grid;
  info->num_splits = pl.ns;
  info->group_warps = pl.ns == 0 ? pl.gsz : 0;
  info->merge_rows_global = pl.wslot_global ? 1 : 0;
  info->merge_pass = post ? 1 : 0;
  info->kernels = p->batch == 0 ? 0 : (post ? 2 : 1);
  info->smem_bytes = pl.smem;
  info->workspace_bytes = pl.ws_bytes;
  info->counter_count = pl.counters;
  info->cluster_size = pl.clu;
  return PA_OK;
}

pa_status_t pa_decode(const pa_decode_params* p, cudaStream_t stream) {
  const pa_status_t v = validate_launch(p);
  if (v != PA_OK) return v;
  const int dev = current_device();
  const int sms = sm_count(dev);
  if (sms <= 0) return PA_ERR_LAUNCH;
  Plan pl;
  pa_status_t s = make_plan(p, sms, pl);
  if (s != PA_OK) return s;
  if (p->batch == 0) return PA_OK;
  if (pl.counters > 0 && (pl.counters > p->counter_count || !p->counters)) return PA_ERR_WORKSPACE;
  if (pl.ws_bytes > p->workspace_bytes || (pl.ws_bytes && !p->workspace)) return PA_ERR_WORKSPACE;
  if (!aligned16(p->workspace)) return PA_ERR_ARG;
  if (pl.generic) return launch_generic(p, pl, stream) == cudaSuccess ? PA_OK : PA_ERR_LAUNCH;

  KParams kp;
  const int tile = kVariants[pl.variant - 1].tile;
  build_kparams(p, pl, kp);

  CUtensorMap mk, mv;
  if (!cached_cache_map(&mk, p, dev, p->k_cache, p->k_stride_block, p->k_stride_slot,
                        p->k_stride_head, kp.R) ||
      !cached_cache_map(&mv, p, dev, p->v_cache, p->v_stride_block, p->v_stride_slot,
                        p->v_stride_head, kp.R))
    return PA_ERR_ARG;

  dim3 merge_grid(1);
  int by_segment = 0, col_split = 0;
  kp.post_merge = want_post_merge(p, pl, kp, merge_grid, by_segment, col_split) ? 1 : 0;
  // A snapped boundary moves by up to half the longest segment, which one CTA
  // then streams on top of its share: only worth it while that is about the
  // cost of the cross-CTA merge it saves (<= 64 KB of K+V, ~1.5 us of one
  // SM's share of HBM). Long segments (B256 log-uniform 512-32K rows: up to
  // 1024 tiles moved, +10 % on the step) keep the token-balanced boundaries.
  const long long seg_bytes = static_cast<long long>(kp.max_nt) * tile * p->head_dim * 4;
  kp.snap = (pl.ns == 0 && pl.use_cum && pl.gsz > 1 && !kp.post_merge &&
             seg_bytes <= (128ll << 10))
                ? 1
                : 0;

  auto launch_decode = [&]() {
    if (p->dtype == PA_F16)
      return pl.dup ? launch<__half, true>(pl, mk, mv, kp, stream, dev)
                    : launch<__half, false>(pl, mk, mv, kp, stream, dev);
    return pl.dup ? launch<__nv_bfloat16, true>(pl, mk, mv, kp, stream, dev)
                  : launch<__nv_bfloat16, false>(pl, mk, mv, kp, stream, dev);
  };
  cudaError_t e = launch_decode();
  if (e == cudaErrorCooperativeLaunchTooLarge && pl.clu) {
    // the clusters cannot all be resident on this device: the plain schedule
    cluster_mark_bad(cluster_key(p, pl));
    pl = Plan();
    s = make_plan(p, sms, pl, false);
    if (s != PA_OK) return s;
    build_kparams(p, pl, kp);
    kp.post_merge = want_post_merge(p, pl, kp, merge_grid, by_segment, col_split) ? 1 : 0;
    e = launch_decode();
  }
  if (e == cudaSuccess && kp.post_merge) {
    MergeParams m;
    memset(&m, 0, sizeof(m));
    m.o_part = kp.o_part;
    m.lse_part = kp.lse_part;
    m.out = kp.out;
    m.o_sb = kp.o_sb;
    m.o_sh = kp.o_sh;
    m.lse = kp.lse;
    m.seq_lens = kp.seq_lens;
    m.cap = kp.max_blocks * kp.bs;
    m.B = kp.B;
    m.Hkv = kp.Hkv;
    m.G = kp.G;
    m.QC = kp.QC;
    m.slot_cols = kp.slot_cols;
    m.tile = tile;
    m.ngroups = pl.W / pl.gsz;
    m.gsz = pl.gsz;
    m.U = kp.U;
    m.P = kp.P;
    m.nt_u = kp.nt_u;
    m.per_row = kp.per_row;
    m.by_segment = by_segment;
    m.col_split = col_split;
    e = p->dtype == PA_F16 ? launch_merge<__half>(m, pl.D, pl.use_cum, merge_grid, stream)
                           : launch_merge<__nv_bfloat16>(m, pl.D, pl.use_cum, merge_grid, stream);
  }
  return e == cudaSuccess ? PA_OK : PA_ERR_LAUNCH;
}

}  // extern "C"

// ----------------------------------------------------------------------------
// Allocation-free entry point: scratch in a file-scope device array
// ----------------------------------------------------------------------------
namespace pa {

// Zero-initialised at module load on every device that loads the library.
static __device__ __align__(256) unsigned char g_noalloc_scratch[PA_NOALLOC_SCRATCH_BYTES];
static void* g_noalloc_addr[64];   // device address of g_noalloc_scratch, per device

// Device address of the scratch array on `dev` (the current device); looked
// up once per device. The host-side symbol is not a device address.
static void* noalloc_scratch(int dev) {
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_noalloc_addr[dev]) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess) return nullptr;
    g_noalloc_addr[dev] = ptr;
  }
  return g_noalloc_addr[dev];
}

}  // namespace pa

extern "C" {

pa_status_t pa_decode_noalloc(const pa_decode_params* p, cudaStream_t stream) {
  // every check pa_decode makes before launching, so that a rejected call
  // queues nothing (not even the counter memset below)
  const pa_status_t v = validate_launch(p);
  if (v != PA_OK) return v;
  const int dev = current_device();
  const int sms = sm_count(dev);
  if (sms <= 0) return PA_ERR_LAUNCH;
  Plan pl;
  const pa_status_t s = make_plan(p, sms, pl);
  if (s != PA_OK) return s;
  const size_t counter_bytes = (pl.counters * sizeof(int32_t) + 255) & ~size_t(255);
  if (counter_bytes + pl.ws_bytes > PA_NOALLOC_SCRATCH_BYTES) return PA_ERR_WORKSPACE;
  if (p->batch == 0) return pa_decode(p, stream);
  unsigned char* base = static_cast<unsigned char*>(noalloc_scratch(dev));
  if (!base) return PA_ERR_LAUNCH;
  // The counters must start at zero; the previous call's partials need no clearing.
  if (counter_bytes && cudaMemsetAsync(base, 0, counter_bytes, stream) != cudaSuccess)
    return PA_ERR_LAUNCH;
  pa_decode_params q = *p;
  q.counters = reinterpret_cast<int32_t*>(base);
  q.counter_count = pl.counters;
  q.workspace = pl.ws_bytes ? base + counter_bytes : nullptr;
  q.workspace_bytes = pl.ws_bytes;
  return pa_decode(&q, stream);
}

pa_status_t pa_cache_append(const pa_append_params* p, cudaStream_t stream) {
  if (!p) return PA_ERR_ARG;
  if (p->num_tokens < 0 || p->num_kv_heads <= 0 || p->head_dim <= 0 || p->block_size <= 0 ||
      p->num_blocks <= 0)
    return PA_ERR_ARG;
  if (p->dtype != PA_F16 && p->dtype != PA_BF16) return PA_ERR_ARG;
  if (p->head_dim % 8) return PA_ERR_UNSUPPORTED;
  if (p->num_tokens == 0) return PA_OK;
  if (!p->key || !p->value || !p->k_cache || !p->v_cache || !p->slot_mapping) return PA_ERR_ARG;
  if (!aligned16(p->key) || !aligned16(p->value) || !aligned16(p->k_cache) ||
      !aligned16(p->v_cache))
    return PA_ERR_ARG;
  const int64_t strides[10] = {p->key_stride_t,   p->key_stride_h,   p->value_stride_t,
                               p->value_stride_h, p->k_stride_block, p->k_stride_slot,
                               p->k_stride_head,  p->v_stride_block, p->v_stride_slot,
                               p->v_stride_head};
  for (int i = 0; i < 10; ++i)
    if (strides[i] % 8) return PA_ERR_ARG;
  const int sms = sm_count(current_device());
  if (sms <= 0) return PA_ERR_LAUNCH;
  AppendParams a;
  a.key = static_cast<const char*>(p->key);
  a.value = static_cast<const char*>(p->value);
  a.k_st = p->key_stride_t * 2;
  a.k_sh = p->key_stride_h * 2;
  a.v_st = p->value_stride_t * 2;
  a.v_sh = p->value_stride_h * 2;
  a.kc = static_cast<char*>(p->k_cache);
  a.vc = static_cast<char*>(p->v_cache);
  a.kc_sb = p->k_stride_block * 2;
  a.kc_ss = p->k_stride_slot * 2;
  a.kc_sh = p->k_stride_head * 2;
  a.vc_sb = p->v_stride_block * 2;
  a.vc_ss = p->v_stride_slot * 2;
  a.vc_sh = p->v_stride_head * 2;
  a.slots = reinterpret_cast<const long long*>(p->slot_mapping);
  a.T = p->num_tokens;
  a.Hkv = p->num_kv_heads;
  a.chunks = p->head_dim / 8;
  a.bs = p->block_size;
  a.NB = p->num_blocks;
  a.status = p->status;
  const long long total = 2ll * p->num_tokens * p->num_kv_heads * a.chunks;
  const long long want = (total + 255) / 256;
  const int grid = static_cast<int>(std::min<long long>(want, 8ll * sms));
  cache_append_kernel<<<grid, 256, 0, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? PA_OK : PA_ERR_LAUNCH;
}

pa_status_t pa_selftest_wait_timeout(const void* src, void* dst, uint64_t limit_ns,
                                     uint32_t* status, cudaStream_t stream) {
  if (!src || !dst || !status || !aligned16(src) || !aligned16(dst)) return PA_ERR_ARG;
  if (limit_ns < 1000ull || limit_ns > 100000000ull) return PA_ERR_ARG;
  wait_timeout_selftest_kernel<<<1, 32, 0, stream>>>(static_cast<const uint4*>(src),
                                                     static_cast<uint4*>(dst), limit_ns, status);
  return cudaGetLastError() == cudaSuccess ? PA_OK : PA_ERR_LAUNCH;
}

pa_status_t pa_stream_copy(const void* src, void* dst, size_t bytes, cudaStream_t stream) {
  if (!src || !dst || (bytes & 15) || !aligned16(src) || !aligned16(dst)) return PA_ERR_ARG;
  const size_t n = bytes / 16;
  const size_t per_cta = static_cast<size_t>(kCopyThreads) * kCopyUnroll;
  const size_t grid = (n + per_cta - 1) / per_cta;
  if (grid == 0) return PA_OK;
  if (grid > 0x7fffffffull) return PA_ERR_ARG;
  stream_copy_kernel<<<static_cast<unsigned>(grid), kCopyThreads, 0, stream>>>(
      static_cast<const uint4*>(src), static_cast<uint4*>(dst), n);
  return cudaGetLastError() == cudaSuccess ? PA_OK : PA_ERR_LAUNCH;
}

pa_status_t pa_stream_read(const void* src, size_t bytes, uint32_t* sink, cudaStream_t stream) {
  if (!src || !sink || (bytes & 15) || !aligned16(src)) return PA_ERR_ARG;
  const int sms = sm_count(current_device());
  if (sms <= 0) return PA_ERR_LAUNCH;
  stream_read_kernel<<<sms * 4, 512, 0, stream>>>(static_cast<const uint4*>(src), bytes / 16,
                                                   sink);
  return cudaGetLastError() == cudaSuccess ? PA_OK : PA_ERR_LAUNCH;
}

}  // extern "C"

#else  // decode-kernel parts (still inside namespace pa)
#if PA_PART == 1
PA_D128(, __half)
#elif PA_PART == 2
PA_D128(, __nv_bfloat16)
#elif PA_PART == 3
PA_D64(, __half)
PA_D64(, __nv_bfloat16)
#elif PA_PART == 4
PA_D256(, __half)
PA_D256(, __nv_bfloat16)
#endif
}  // namespace pa
#endif  // PA_HOST_PART
