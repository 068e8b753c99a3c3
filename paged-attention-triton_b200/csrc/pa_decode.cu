// pa_decode.cu -- paged-attention decode for B200 (sm_100a).
//
// One persistent kernel per decode step. Each warp is an independent worker:
// it owns a contiguous range of 32-token tiles of the flattened
// (sequence, kv-head, tile) space, streams the K/V page rows of those tiles
// into shared memory with TMA (cp.async.bulk.tensor, 128-byte swizzle, a
// 3-deep mbarrier ring per warp), and runs the FP32 online softmax with both
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

namespace pa {

constexpr int kD = 128;             // head_dim
constexpr int kTile = 32;           // tokens per pipeline stage
constexpr int kWarps = 4;           // worker warps per CTA
constexpr int kStages = 3;          // ring depth per worker
constexpr int kHalfBytes = kTile * 128;          // one 64-dim half of a K or V tile
constexpr int kKVBytes = 2 * kHalfBytes;         // one K (or V) tile: 8 KB
constexpr int kQBytes = 8 * kD * 2;              // up to 8 query heads
constexpr int kStageBytes = 2 * kKVBytes + kQBytes;   // 18 KB, multiple of 1 KB
constexpr int kCumMax = 2048;       // rows whose tile prefix sum fits in shared memory
constexpr int kSmemBytes = kWarps * kStages * kStageBytes + (kCumMax + 1) * 4 + 1024 + 128;
constexpr float kSentinel = -1e30f;     // split_kv_kernel.py:8
constexpr float kValidLse = -1e29f;     // split_kv_kernel.py:9
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr unsigned long long kWaitLimitNs = 2000000000ull;   // 2 s per barrier wait
constexpr unsigned kFull = 0xffffffffu;

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
  int seq_len;              // clamped uniform length (seq_lens == nullptr)
  int B, Hq, Hkv, G, QC, bs, NB;
  int nseg;                 // Hkv * QC segments per row
  int ns;                   // 0: balanced schedule
  float scale_log2;
  float* o_part;            // split: [B, Hq, ns, D]; balanced: [2W, 8, D]
  float* lse_part;          // split: [B, Hq, ns];    balanced: [2W, 8]
  int* counters;
  unsigned* status;
  int R;                    // rows per TMA box (gcd(bs, kTile))
  int spt;                  // boxes per tile (kTile / R)
  int W;                    // workers
  int use_cum;              // balanced + seq_lens: prefix sums in shared memory
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
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - t0 > kWaitLimitNs) return false;
  }
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, int c3, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
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
};

__device__ __forceinline__ uint32_t pack16(uint16_t lo, uint16_t hi) {
  return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

// ----------------------------------------------------------------------------
// Work decomposition
// ----------------------------------------------------------------------------
struct Tile {
  int b, seg, tile;   // row, segment within the row (kvh * QC + qc), tile within the segment
  int t0, t1;         // token range of this worker's piece of the segment
  int seg_lo, seg_hi; // unit range of the segment (balanced) / split index in seg_lo (split)
  bool first, last, whole;
};

struct Work {
  int n;                // tiles of this worker
  int u0, u1;           // balanced: unit range
  int per;              // balanced: units per worker
  int b, seg, s, t0, t1;  // split: the one piece
};

__device__ __forceinline__ int clamp_len(const KParams& p, int s, bool& bad) {
  const int cap = p.max_blocks * p.bs;
  if (s < 0) { bad = true; return 0; }
  if (s > cap) { bad = true; return cap; }
  return s;
}

__device__ __forceinline__ int row_len(const KParams& p, int b) {
  if (p.seq_lens == nullptr) return p.seq_len;
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

__device__ __forceinline__ void get_tile(const KParams& p, const int* cum, const Work& w, int i,
                                         Tile& t) {
  if (p.ns == 0) {
    const int u = w.u0 + i;
    int b, base, S, nt;
    if (p.use_cum) {
      b = find_row(cum, p.B, u);
      base = cum[b];
      S = row_len(p, b);
      nt = (S + kTile - 1) / kTile;
    } else {
      S = p.seq_len;
      nt = (S + kTile - 1) / kTile;
      const int per_row = p.nseg * nt;
      b = u / per_row;
      base = b * per_row;
    }
    const int r = u - base;
    t.b = b;
    t.seg = r / nt;
    t.tile = r - t.seg * nt;
    t.seg_lo = base + t.seg * nt;
    t.seg_hi = t.seg_lo + nt;
    const int plo = max(t.seg_lo, w.u0), phi = min(t.seg_hi, w.u1);
    t.first = (u == plo);
    t.last = (u == phi - 1);
    t.whole = (plo == t.seg_lo) && (phi == t.seg_hi);
    t.t0 = (plo - t.seg_lo) * kTile;
    t.t1 = min(S, (phi - t.seg_lo) * kTile);
  } else {
    t.b = w.b;
    t.seg = w.seg;
    t.tile = w.t0 / kTile + i;
    t.t0 = w.t0;
    t.t1 = w.t1;
    t.seg_lo = w.s;
    t.seg_hi = 0;
    t.first = (i == 0);
    t.last = (i == w.n - 1);
    t.whole = false;
  }
}

// Physical block of this lane's TMA box in window `win`, or INT_MIN when the box
// holds no token of the piece (never loaded, masked by the consumer).
__device__ __forceinline__ int fetch_window(const KParams& p, const int* cum, const Work& w, int win,
                                            int lane, int wt) {
  const int i = win * wt + lane / p.spt;
  if (i >= w.n) return INT_MIN;
  Tile t;
  get_tile(p, cum, w, i, t);
  const int tt = t.tile * kTile + (lane % p.spt) * p.R;
  if (tt >= t.t1 || tt + p.R <= t.t0) return INT_MIN;
  return __ldg(p.bt + static_cast<long long>(t.b) * p.bt_sb + tt / p.bs);
}

__device__ __forceinline__ void flag(const KParams& p, unsigned bits) {
  if (p.status) atomicOr(p.status, bits);
}

// ----------------------------------------------------------------------------
// Kernel
// ----------------------------------------------------------------------------
template <typename T, bool kDup>
__global__ void __launch_bounds__(kWarps * 32, 1)
    pa_decode_kernel(const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const KParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kWarps * kStages * kStageBytes);
  int* cum = reinterpret_cast<int*>(bars + kWarps * kStages);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmK)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmV)) : "memory");
  }
  if (lane == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(smem_u32(&bars[warp * kStages + s]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }

  // Balanced schedule with per-row lengths: per-row tile prefix sums.
  if (p.ns == 0 && p.use_cum) {
    const int B = p.B;
    const int chunk = (B + blockDim.x - 1) / blockDim.x;
    const int lo = min(B, static_cast<int>(threadIdx.x) * chunk);
    const int hi = min(B, lo + chunk);
    bool bad = false;
    int local = 0;
    for (int b = lo; b < hi; ++b) {
      const int S = clamp_len(p, __ldg(p.seq_lens + b), bad);
      local += p.nseg * ((S + kTile - 1) / kTile);
    }
    if (bad && blockIdx.x == 0) flag(p, PA_STATUS_BAD_SEQLEN);
    // exclusive scan of `local` over the block
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += v;
    }
    __shared__ int warp_tot[kWarps];
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    int before = 0;
    for (int k = 0; k < warp; ++k) before += warp_tot[k];
    int run = before + incl - local;
    for (int b = lo; b < hi; ++b) {
      cum[b] = run;
      const int S = clamp_len(p, __ldg(p.seq_lens + b), bad);
      run += p.nseg * ((S + kTile - 1) / kTile);
    }
    if (threadIdx.x == blockDim.x - 1) cum[B] = before + incl;
  }
  __syncthreads();

  // Rows of length 0 own no tile: O = 0 and LSE = -1e30 (split_kv_kernel.py:101,120).
  if (p.ns == 0) {
    for (int b = blockIdx.x; b < p.B; b += gridDim.x) {
      if (row_len(p, b) != 0) continue;
      for (int idx = threadIdx.x; idx < p.Hq * (kD / 8); idx += blockDim.x) {
        const int h = idx / (kD / 8), c = idx % (kD / 8);
        *reinterpret_cast<uint4*>(p.out + b * p.o_sb + h * p.o_sh + c * 16) =
            make_uint4(0, 0, 0, 0);
      }
      if (p.lse)
        for (int h = threadIdx.x; h < p.Hq; h += blockDim.x) p.lse[b * p.Hq + h] = kSentinel;
    }
  }

  // ---------------------------------------------------------------- my work
  const int wid = warp * gridDim.x + blockIdx.x;
  Work w;
  if (p.ns == 0) {
    const int U = p.use_cum ? cum[p.B] : p.B * p.nseg * ((p.seq_len + kTile - 1) / kTile);
    w.per = max(1, (U + p.W - 1) / p.W);
    w.u0 = min(U, wid * w.per);
    w.u1 = min(U, w.u0 + w.per);
    w.n = w.u1 - w.u0;
  } else {
    const int total = p.B * p.nseg * p.ns;
    if (wid >= total) return;
    w.s = wid % p.ns;
    const int rs = wid / p.ns;
    w.seg = rs % p.nseg;
    w.b = rs / p.nseg;
    bool bad = false;
    const int S = p.seq_lens ? clamp_len(p, __ldg(p.seq_lens + w.b), bad) : p.seq_len;
    if (bad && w.s == 0 && w.seg == 0) flag(p, PA_STATUS_BAD_SEQLEN);
    const int ss = (S + p.ns - 1) / p.ns;       // torch_kernel.py:30
    w.t0 = w.s * ss;
    w.t1 = min(w.t0 + ss, S);
    w.n = (w.t0 < w.t1) ? ((w.t1 - 1) / kTile - w.t0 / kTile + 1) : 0;
  }

  const uint32_t stage0 = smem_u32(smem + warp * kStages * kStageBytes);
  const uint32_t bar0 = smem_u32(&bars[warp * kStages]);
  const int wt = 32 / p.spt;  // tiles per page-index window

  // Output-side helpers.
  const int G = p.G;
  auto seg_heads = [&](int seg, int& kvh, int& qc, int& gc) {
    kvh = seg / p.QC;
    qc = seg - kvh * p.QC;
    gc = min(8, G - qc * 8);
  };

  if (p.ns != 0 && w.n == 0) {
    // Empty split (split_kv_kernel.py:32-33): partial LSE keeps the sentinel.
    int kvh, qc, gc;
    seg_heads(w.seg, kvh, qc, gc);
    for (int j = 0; j < gc; ++j) {
      const int hq = kvh * G + qc * 8 + j;
      const long long row = (static_cast<long long>(w.b) * p.Hq + hq) * p.ns + w.s;
      for (int d = lane; d < kD; d += 32) p.o_part[row * kD + d] = 0.f;
      if (lane == 0) p.lse_part[row] = kSentinel;
    }
    __threadfence();
    __syncwarp();
    int last = 0;
    const int cid = (w.b * p.Hkv + kvh) * p.QC + qc;
    if (lane == 0) last = (atomicAdd(p.counters + cid, 1) == p.ns - 1);
    last = __shfl_sync(kFull, last, 0);
    if (!last) return;
    __threadfence();
    // fall through to the merge below with an empty tile list
  }

  // Page-index windows (register double buffer, one entry per lane).
  int win = 0;
  int pg_cur = w.n > 0 ? fetch_window(p, cum, w, 0, lane, wt) : INT_MIN;
  int pg_nxt = w.n > wt ? fetch_window(p, cum, w, 1, lane, wt) : INT_MIN;

  auto issue = [&](int i, int st) {
    if (i / wt != win) {
      ++win;
      pg_cur = pg_nxt;
      pg_nxt = fetch_window(p, cum, w, win + 1, lane, wt);
    }
    Tile t;
    get_tile(p, cum, w, i, t);
    int kvh, qc, gc;
    seg_heads(t.seg, kvh, qc, gc);
    const bool mine = (lane / p.spt) == (i % wt);
    bool valid = mine && pg_cur != INT_MIN;
    if (valid && (pg_cur < 0 || pg_cur >= p.NB)) {
      flag(p, PA_STATUS_BAD_BLOCK);
      valid = false;
    }
    const unsigned vm = __ballot_sync(kFull, valid);
    const uint32_t bar = bar0 + st * 8;
    const uint32_t qbytes = t.first ? gc * kD * 2 : 0;
    if (lane == 0) mbar_expect_tx(bar, __popc(vm) * 4 * p.R * 128 + qbytes);
    __syncwarp();
    const uint32_t sk = stage0 + st * kStageBytes;
    if (valid) {
      const int j = lane % p.spt;
      const int tt = t.tile * kTile + j * p.R;
      const int slot = tt % p.bs;
      const uint32_t row_off = j * p.R * 128;
      tma_load_4d(sk + row_off, &tmK, 0, kvh, slot, pg_cur, bar);
      tma_load_4d(sk + kHalfBytes + row_off, &tmK, 64, kvh, slot, pg_cur, bar);
      tma_load_4d(sk + kKVBytes + row_off, &tmV, 0, kvh, slot, pg_cur, bar);
      tma_load_4d(sk + kKVBytes + kHalfBytes + row_off, &tmV, 64, kvh, slot, pg_cur, bar);
    }
    if (t.first && lane < gc) {
      const int hq = kvh * G + qc * 8 + lane;
      bulk_load(sk + 2 * kKVBytes + lane * kD * 2, p.q + t.b * p.q_sb + hq * p.q_sh, kD * 2, bar);
    }
  };

  const int npro = min(kStages, w.n);
  for (int i = 0; i < npro; ++i) issue(i, i);

  // Consumer state.
  uint32_t qf[8][2];
  float acc[8][4];
  float m_run[2], l_run[2];
  uint32_t phase = 0;
  bool aborted = false;

  const int qd = lane & 3;     // column pair index: columns 2*qd, 2*qd+1
  const int rr = lane >> 2;    // fragment row

  for (int i = 0; i < w.n; ++i) {
    const int st = i % kStages;
    Tile t;
    get_tile(p, cum, w, i, t);
    int kvh, qc, gc;
    seg_heads(t.seg, kvh, qc, gc);
    const uint32_t sk = stage0 + st * kStageBytes;
    const uint32_t sv = sk + kKVBytes;
    const uint32_t sq = sk + 2 * kKVBytes;

    if (!mbar_wait(bar0 + st * 8, (phase >> st) & 1)) {
      flag(p, PA_STATUS_TIMEOUT);
      aborted = true;
      // drain the copies still in flight for the other stages (bounded)
      for (int k = i + 1; k < min(w.n, i + kStages); ++k)
        mbar_wait(bar0 + (k % kStages) * 8, (phase >> (k % kStages)) & 1);
      break;
    }
    phase ^= 1u << st;

    if (t.first) {
      // Query fragments (B operand of S^T = K Q^T): column n -> query head.
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int n = rr;
          int head;
          if (kDup) head = (n < 2 * gc) ? (n % gc) : -1;
          else head = (n < gc) ? n : -1;
          uint32_t v = 0;
          if (head >= 0) {
            const uint32_t addr = sq + head * kD * 2 + (ks * 16 + h * 8 + qd * 2) * 2;
            asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
          }
          qf[ks][h] = v;
        }
      }
#pragma unroll
      for (int md = 0; md < 8; ++md)
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[md][r] = 0.f;
      m_run[0] = m_run[1] = -INFINITY;
      l_run[0] = l_run[1] = 0.f;
    }

    // ---- S^T = K Q^T: 32 tokens x 8 query columns, FP32 accumulate.
    float s[2][4];
#pragma unroll
    for (int mb = 0; mb < 2; ++mb) {
#pragma unroll
      for (int r = 0; r < 4; ++r) s[mb][r] = 0.f;
      const int row = mb * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int c = ks * 2 + (lane >> 4);
        const uint32_t addr =
            sk + (c >> 3) * kHalfBytes + row * 128 + (((c & 7) ^ (lane & 7)) << 4);
        uint32_t a[4];
        ldsm_x4(addr, a);
        Mma<T>::run(s[mb], a, qf[ks][0], qf[ks][1]);
      }
    }

    // ---- mask, scale, online softmax (split_kv_kernel.py:68-77).
    const int tb = t.tile * kTile;
    const bool partial = (t.t0 > tb) || (t.t1 < tb + kTile);
#pragma unroll
    for (int mb = 0; mb < 2; ++mb)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        float v = s[mb][r] * p.scale_log2;
        if (partial) {
          const int tok = tb + mb * 16 + rr + (r >> 1) * 8;
          if (tok < t.t0 || tok >= t.t1) v = -INFINITY;
        }
        s[mb][r] = v;
      }
    float alpha[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float mx = fmaxf(fmaxf(s[0][e], s[0][e + 2]), fmaxf(s[1][e], s[1][e + 2]));
      mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 4));
      mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 16));
      const float mn = fmaxf(m_run[e], mx);
      alpha[e] = exp2f(m_run[e] - mn);
      m_run[e] = mn;
    }
    float psum[2] = {0.f, 0.f};
#pragma unroll
    for (int mb = 0; mb < 2; ++mb)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const float pv = exp2f(s[mb][r] - m_run[r & 1]);
        s[mb][r] = pv;
        psum[r & 1] += pv;
      }
#pragma unroll
    for (int e = 0; e < 2; ++e) l_run[e] = l_run[e] * alpha[e] + psum[e];
#pragma unroll
    for (int md = 0; md < 8; ++md) {
      acc[md][0] *= alpha[0];
      acc[md][1] *= alpha[1];
      acc[md][2] *= alpha[0];
      acc[md][3] *= alpha[1];
    }

    // ---- P^T as the B operand: hi/lo split keeps ~16 (bf16) / 22 (fp16) bits of p.
    uint32_t bh[2][2], bl[2][2];
#pragma unroll
    for (int kb = 0; kb < 2; ++kb) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint16_t hi0, lo0, hi1, lo1;
        Mma<T>::split(s[kb][half * 2 + 0], hi0, lo0);
        Mma<T>::split(s[kb][half * 2 + 1], hi1, lo1);
        const int c0 = qd * 2, c1 = qd * 2 + 1;
        if (kDup) {
          const uint16_t v0 = c0 < gc ? hi0 : (c0 < 2 * gc ? lo0 : uint16_t(0));
          const uint16_t v1 = c1 < gc ? hi1 : (c1 < 2 * gc ? lo1 : uint16_t(0));
          bh[kb][half] = movm_trans(pack16(v0, v1));
        } else {
          bh[kb][half] = movm_trans(pack16(c0 < gc ? hi0 : 0, c1 < gc ? hi1 : 0));
          bl[kb][half] = movm_trans(pack16(c0 < gc ? lo0 : 0, c1 < gc ? lo1 : 0));
        }
      }
    }

    // ---- O^T += V^T P^T (dims x columns).
#pragma unroll
    for (int kb = 0; kb < 2; ++kb) {
      uint32_t m01 = 0xffffffffu, m23 = 0xffffffffu;
      if (partial) {
        const int tk = tb + kb * 16 + qd * 2;
        auto ok = [&](int x) { return x >= t.t0 && x < t.t1; };
        m01 = (ok(tk) ? 0x0000ffffu : 0u) | (ok(tk + 1) ? 0xffff0000u : 0u);
        m23 = (ok(tk + 8) ? 0x0000ffffu : 0u) | (ok(tk + 9) ? 0xffff0000u : 0u);
      }
      const int row = kb * 16 + (lane >> 4) * 8 + (lane & 7);
#pragma unroll
      for (int md = 0; md < 8; ++md) {
        const int c = md * 2 + ((lane >> 3) & 1);
        const uint32_t addr =
            sv + (c >> 3) * kHalfBytes + row * 128 + (((c & 7) ^ (lane & 7)) << 4);
        uint32_t a[4];
        ldsm_x4_t(addr, a);
        a[0] &= m01;
        a[1] &= m01;
        a[2] &= m23;
        a[3] &= m23;
        Mma<T>::run(acc[md], a, bh[kb][0], bh[kb][1]);
        if (!kDup) Mma<T>::run(acc[md], a, bl[kb][0], bl[kb][1]);
      }
    }

    __syncwarp();
    if (i + kStages < w.n) issue(i + kStages, st);

    if (!t.last) continue;

    // ---------------------------------------------------------- piece epilogue
    float lsum[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float v = l_run[e];
      v += __shfl_xor_sync(kFull, v, 4);
      v += __shfl_xor_sync(kFull, v, 8);
      v += __shfl_xor_sync(kFull, v, 16);
      lsum[e] = v;
    }
    // Combine hi/lo columns (dup layout): column c + gc holds the low part of c.
    float o[8][4];
#pragma unroll
    for (int md = 0; md < 8; ++md)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        float v = acc[md][r];
        if (kDup) {
          float partner;
          if (gc == 1) {
            partner = acc[md][r | 1];
          } else {
            partner = __shfl_down_sync(kFull, v, gc >> 1);
          }
          v += partner;
        }
        o[md][r] = v;
      }

    // Where this piece's normalised output and LSE go.
    const bool final_out = (p.ns == 0) && t.whole;
    long long slot_row = 0;    // split: row of [B*Hq*ns]; balanced: slot
    int n_pieces = 0, w_first = 0;
    if (p.ns == 0 && !final_out) {
      w_first = t.seg_lo / w.per;
      const int w_last = (t.seg_hi - 1) / w.per;
      n_pieces = w_last - w_first + 1;
      const int plo = max(t.seg_lo, w.u0);
      slot_row = 2ll * wid + (plo == w.u0 ? 0 : 1);
    }
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int c = qd * 2 + e;
      if (c >= gc) continue;
      const int hq = kvh * G + qc * 8 + c;
      const float inv_l = 1.f / fmaxf(lsum[e], 1e-20f);
      const float lse = (m_run[e] + log2f(fmaxf(lsum[e], 1e-20f))) * kLn2;
      if (final_out) {
        char* dst = p.out + t.b * p.o_sb + hq * p.o_sh;
#pragma unroll
        for (int md = 0; md < 8; ++md) {
          const int d0 = md * 16 + rr;
          *reinterpret_cast<uint16_t*>(dst + d0 * 2) = Mma<T>::from_float(o[md][e] * inv_l);
          *reinterpret_cast<uint16_t*>(dst + (d0 + 8) * 2) =
              Mma<T>::from_float(o[md][e + 2] * inv_l);
        }
        if (rr == 0 && p.lse) p.lse[t.b * p.Hq + hq] = lse;
      } else {
        float* od;
        float* ld;
        if (p.ns == 0) {
          od = p.o_part + (slot_row * 8 + c) * kD;
          ld = p.lse_part + slot_row * 8 + c;
        } else {
          const long long row = (static_cast<long long>(t.b) * p.Hq + hq) * p.ns + t.seg_lo;
          od = p.o_part + row * kD;
          ld = p.lse_part + row;
        }
#pragma unroll
        for (int md = 0; md < 8; ++md) {
          const int d0 = md * 16 + rr;
          od[d0] = o[md][e] * inv_l;
          od[d0 + 8] = o[md][e + 2] * inv_l;
        }
        if (rr == 0) *ld = lse;
      }
    }
    if (final_out) continue;

    // Publish the partial; the last arriving piece merges the segment.
    __threadfence();
    __syncwarp();
    const int n_expect = (p.ns == 0) ? n_pieces : p.ns;
    const int cid = (t.b * p.Hkv + kvh) * p.QC + qc;
    int last = 0;
    if (lane == 0) last = (atomicAdd(p.counters + cid, 1) == n_expect - 1);
    last = __shfl_sync(kFull, last, 0);
    if (!last) continue;
    __threadfence();

    // ------------------------------------------------------ merge (last arriver)
    // split_kv_kernel.py:101-122: skip lse <= -1e29, running max, divide by
    // max(sum, 1e-20). Each lane owns 4 dims.
    for (int j = 0; j < gc; ++j) {
      const int hq = kvh * G + qc * 8 + j;
      auto part = [&](int k, const float*& op, const float*& lp) {
        if (p.ns == 0) {
          const int wk = w_first + k;
          const int plo = max(t.seg_lo, wk * w.per);
          const long long sl = 2ll * wk + (plo == wk * w.per ? 0 : 1);
          op = p.o_part + (sl * 8 + j) * kD;
          lp = p.lse_part + sl * 8 + j;
        } else {
          const long long row = (static_cast<long long>(t.b) * p.Hq + hq) * p.ns + k;
          op = p.o_part + row * kD;
          lp = p.lse_part + row;
        }
      };
      float gmax = kValidLse;
      for (int k = lane; k < n_expect; k += 32) {
        const float* op;
        const float* lp;
        part(k, op, lp);
        const float l = __ldcg(lp);
        if (l > kValidLse) gmax = fmaxf(gmax, l);
      }
#pragma unroll
      for (int o2 = 16; o2 > 0; o2 >>= 1) gmax = fmaxf(gmax, __shfl_xor_sync(kFull, gmax, o2));
      float4 a4 = make_float4(0.f, 0.f, 0.f, 0.f);
      float gsum = 0.f;
      for (int k = 0; k < n_expect; ++k) {
        const float* op;
        const float* lp;
        part(k, op, lp);
        const float l = __ldcg(lp);
        if (!(l > kValidLse)) continue;
        const float wgt = exp2f((l - gmax) * kLog2e);
        const float4 v = __ldcg(reinterpret_cast<const float4*>(op) + lane);
        a4.x += wgt * v.x;
        a4.y += wgt * v.y;
        a4.z += wgt * v.z;
        a4.w += wgt * v.w;
        gsum += wgt;
      }
      const float inv = 1.f / fmaxf(gsum, 1e-20f);
      char* dst = p.out + t.b * p.o_sb + hq * p.o_sh + lane * 8;
      const uint32_t lo = pack16(Mma<T>::from_float(a4.x * inv), Mma<T>::from_float(a4.y * inv));
      const uint32_t hi = pack16(Mma<T>::from_float(a4.z * inv), Mma<T>::from_float(a4.w * inv));
      *reinterpret_cast<uint2*>(dst) = make_uint2(lo, hi);
      if (lane == 0 && p.lse)
        p.lse[t.b * p.Hq + hq] = gsum > 0.f ? gmax + logf(gsum) : kSentinel;
    }
    if (lane == 0) atomicExch(p.counters + cid, 0);
  }

  // Split schedule, empty piece that arrived last: merge with no tiles of its own.
  if (p.ns != 0 && w.n == 0) {
    int kvh, qc, gc;
    seg_heads(w.seg, kvh, qc, gc);
    for (int j = 0; j < gc; ++j) {
      const int hq = kvh * G + qc * 8 + j;
      const long long row0 = (static_cast<long long>(w.b) * p.Hq + hq) * p.ns;
      float gmax = kValidLse;
      for (int k = lane; k < p.ns; k += 32) {
        const float l = __ldcg(p.lse_part + row0 + k);
        if (l > kValidLse) gmax = fmaxf(gmax, l);
      }
#pragma unroll
      for (int o2 = 16; o2 > 0; o2 >>= 1) gmax = fmaxf(gmax, __shfl_xor_sync(kFull, gmax, o2));
      float4 a4 = make_float4(0.f, 0.f, 0.f, 0.f);
      float gsum = 0.f;
      for (int k = 0; k < p.ns; ++k) {
        const float l = __ldcg(p.lse_part + row0 + k);
        if (!(l > kValidLse)) continue;
        const float wgt = exp2f((l - gmax) * kLog2e);
        const float4 v = __ldcg(reinterpret_cast<const float4*>(p.o_part + (row0 + k) * kD) + lane);
        a4.x += wgt * v.x;
        a4.y += wgt * v.y;
        a4.z += wgt * v.z;
        a4.w += wgt * v.w;
        gsum += wgt;
      }
      const float inv = 1.f / fmaxf(gsum, 1e-20f);
      char* dst = p.out + w.b * p.o_sb + hq * p.o_sh + lane * 8;
      const uint32_t lo = pack16(Mma<T>::from_float(a4.x * inv), Mma<T>::from_float(a4.y * inv));
      const uint32_t hi = pack16(Mma<T>::from_float(a4.z * inv), Mma<T>::from_float(a4.w * inv));
      *reinterpret_cast<uint2*>(dst) = make_uint2(lo, hi);
      if (lane == 0 && p.lse)
        p.lse[w.b * p.Hq + hq] = gsum > 0.f ? gmax + logf(gsum) : kSentinel;
    }
    if (lane == 0) atomicExch(p.counters + (w.b * p.Hkv + kvh) * p.QC + qc, 0);
  }
  (void)aborted;
}

// ----------------------------------------------------------------------------
// Bandwidth probes (replace measure_peak_bw.py:15-21's Triton copy kernel)
// ----------------------------------------------------------------------------
__global__ void __launch_bounds__(512) stream_copy_kernel(const uint4* __restrict__ src,
                                                          uint4* __restrict__ dst, size_t n) {
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (; i + 3 * stride < n; i += 4 * stride) {
    const uint4 a = __ldcs(src + i);
    const uint4 b = __ldcs(src + i + stride);
    const uint4 c = __ldcs(src + i + 2 * stride);
    const uint4 d = __ldcs(src + i + 3 * stride);
    __stcs(dst + i, a);
    __stcs(dst + i + stride, b);
    __stcs(dst + i + 2 * stride, c);
    __stcs(dst + i + 3 * stride, d);
  }
  for (; i < n; i += stride) __stcs(dst + i, __ldcs(src + i));
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
// Host side
// ----------------------------------------------------------------------------
struct DeviceInfo {
  int sms = 0;
  bool attr_set[4] = {false, false, false, false};
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

struct Plan {
  int ns = 0;        // 0: balanced
  int grid = 0;
  int W = 0;
  int G = 1, QC = 1;
  bool use_cum = false;
  size_t ws_bytes = 0;
  size_t counters = 0;
};

static pa_status_t validate(const pa_decode_params* p) {
  if (!p) return PA_ERR_ARG;
  if (p->batch < 0 || p->num_heads <= 0 || p->num_kv_heads <= 0 || p->block_size <= 0 ||
      p->num_blocks <= 0 || p->max_blocks < 0)
    return PA_ERR_ARG;
  if (p->num_heads % p->num_kv_heads != 0) return PA_ERR_ARG;
  if (p->dtype != PA_F16 && p->dtype != PA_BF16) return PA_ERR_ARG;
  if (p->num_splits < 0) return PA_ERR_ARG;
  if (p->seq_lens == nullptr && p->seq_len < 0) return PA_ERR_ARG;
  if (p->seq_lens == nullptr && static_cast<long long>(p->seq_len) >
                                    static_cast<long long>(p->max_blocks) * p->block_size)
    return PA_ERR_ARG;
  if (p->head_dim != kD) return PA_ERR_UNSUPPORTED;
  if (p->block_size % 8 != 0 || p->block_size > (1 << 20)) return PA_ERR_UNSUPPORTED;
  return PA_OK;
}

static pa_status_t make_plan(const pa_decode_params* p, int sms, Plan& pl) {
  pl.G = p->num_heads / p->num_kv_heads;
  pl.QC = (pl.G + 7) / 8;
  const long long nseg = static_cast<long long>(p->num_kv_heads) * pl.QC;
  const long long cap = static_cast<long long>(p->max_blocks) * p->block_size;
  pl.ns = p->num_splits;
  if (pl.ns == 0) {
    const long long nt = (cap + kTile - 1) / kTile;
    // Unit indices must fit int32; very large batches with per-row lengths
    // use the split schedule with the reference heuristic instead.
    if ((p->seq_lens != nullptr && p->batch > kCumMax) ||
        static_cast<long long>(p->batch) * nseg * nt > 0x7fffffffll) {
      const int s_max = static_cast<int>(cap > 0x7fffffff ? 0x7fffffff : cap);
      pl.ns = pa_num_splits_heuristic(p->batch, p->num_heads, s_max, p->block_size, sms);
    }
  }
  if (pl.ns == 0) {
    pl.grid = sms;
    pl.W = pl.grid * kWarps;
    pl.use_cum = p->seq_lens != nullptr;
    pl.ws_bytes = static_cast<size_t>(2) * pl.W * 8 * (kD + 1) * sizeof(float);
  } else {
    const long long workers = static_cast<long long>(p->batch) * nseg * pl.ns;
    if (workers > 0x7fffffffll) return PA_ERR_UNSUPPORTED;
    pl.W = static_cast<int>(workers);
    pl.grid = static_cast<int>((workers + kWarps - 1) / kWarps);
    const size_t rows = static_cast<size_t>(p->batch) * p->num_heads * pl.ns;
    pl.ws_bytes = (p->o_partial && p->lse_partial) ? 0 : rows * (kD + 1) * sizeof(float);
  }
  pl.counters = static_cast<size_t>(p->batch) * nseg;
  return PA_OK;
}

static bool encode_cache_map(CUtensorMap* map, const pa_decode_params* p, const void* base,
                             int64_t s_block, int64_t s_slot, int64_t s_head, int rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  const CUtensorMapDataType dt =
      p->dtype == PA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(p->num_kv_heads),
                        static_cast<cuuint64_t>(p->block_size),
                        static_cast<cuuint64_t>(p->num_blocks)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(s_head) * 2, static_cast<cuuint64_t>(s_slot) * 2,
                           static_cast<cuuint64_t>(s_block) * 2};
  cuuint32_t box[4] = {64, 1, static_cast<cuuint32_t>(rows), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = fn(map, dt, 4, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

static bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; }

template <typename T, bool kDup>
static cudaError_t launch(const Plan& pl, const CUtensorMap& mk, const CUtensorMap& mv,
                          const KParams& kp, cudaStream_t stream, int dev, int attr_idx) {
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_dev[dev].attr_set[attr_idx]) {
      const cudaError_t e = cudaFuncSetAttribute(
          pa_decode_kernel<T, kDup>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
      if (e != cudaSuccess) return e;
      g_dev[dev].attr_set[attr_idx] = true;
    }
  }
  pa_decode_kernel<T, kDup><<<pl.grid, kWarps * 32, kSmemBytes, stream>>>(mk, mv, kp);
  return cudaGetLastError();
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

pa_status_t pa_decode(const pa_decode_params* p, cudaStream_t stream) {
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
  const int dev = current_device();
  const int sms = sm_count(dev);
  if (sms <= 0) return PA_ERR_LAUNCH;
  Plan pl;
  pa_status_t s = make_plan(p, sms, pl);
  if (s != PA_OK) return s;
  if (p->batch == 0) return PA_OK;
  if (pl.counters > p->counter_count || !p->counters) return PA_ERR_WORKSPACE;
  if (pl.ws_bytes > p->workspace_bytes || (pl.ws_bytes && !p->workspace)) return PA_ERR_WORKSPACE;
  if (!aligned16(p->workspace)) return PA_ERR_ARG;

  KParams kp;
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
  kp.nseg = p->num_kv_heads * pl.QC;
  kp.ns = pl.ns;
  kp.scale_log2 = p->scale * kLog2e;
  if (pl.ns == 0) {
    float* ws = static_cast<float*>(p->workspace);
    kp.o_part = ws;
    kp.lse_part = ws + static_cast<size_t>(2) * pl.W * 8 * kD;
  } else if (p->o_partial && p->lse_partial) {
    kp.o_part = p->o_partial;
    kp.lse_part = p->lse_partial;
  } else {
    float* ws = static_cast<float*>(p->workspace);
    const size_t rows = static_cast<size_t>(p->batch) * p->num_heads * pl.ns;
    kp.o_part = ws;
    kp.lse_part = ws + rows * kD;
  }
  kp.counters = p->counters;
  kp.status = p->status;
  kp.R = gcd_int(p->block_size, kTile);
  kp.spt = kTile / kp.R;
  kp.W = pl.W;
  kp.use_cum = pl.use_cum ? 1 : 0;

  CUtensorMap mk, mv;
  if (!encode_cache_map(&mk, p, p->k_cache, p->k_stride_block, p->k_stride_slot, p->k_stride_head,
                        kp.R) ||
      !encode_cache_map(&mv, p, p->v_cache, p->v_stride_block, p->v_stride_slot, p->v_stride_head,
                        kp.R))
    return PA_ERR_ARG;

  const bool dup = (pl.G == 1 || pl.G == 2 || pl.G == 4);
  cudaError_t e;
  if (p->dtype == PA_F16)
    e = dup ? launch<__half, true>(pl, mk, mv, kp, stream, dev, 0)
            : launch<__half, false>(pl, mk, mv, kp, stream, dev, 1);
  else
    e = dup ? launch<__nv_bfloat16, true>(pl, mk, mv, kp, stream, dev, 2)
            : launch<__nv_bfloat16, false>(pl, mk, mv, kp, stream, dev, 3);
  return e == cudaSuccess ? PA_OK : PA_ERR_LAUNCH;
}

pa_status_t pa_stream_copy(const void* src, void* dst, size_t bytes, cudaStream_t stream) {
  if (!src || !dst || (bytes & 15) || !aligned16(src) || !aligned16(dst)) return PA_ERR_ARG;
  const int sms = sm_count(current_device());
  if (sms <= 0) return PA_ERR_LAUNCH;
  stream_copy_kernel<<<sms * 4, 512, 0, stream>>>(static_cast<const uint4*>(src),
                                                   static_cast<uint4*>(dst), bytes / 16);
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
