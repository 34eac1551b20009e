// gather_gemm.cu -- step 2 of the sparse front end: sparse patchify as a
// gather-GEMM, the operation burn_flex_gmm::cuda::sparse_patchify3d_forward_cuda
// performs for burn_jepa (called at src/model.rs:1140, 1197, 1319):
//
//   out[m, d] = bias[d] + sum_k W[d, k] * A[m, k]
//   A[m, k]   = x[b, c, t*kt + dt, r*ph + dy, col*pw + dx],  (b, t, r, col) = coords[m]
//   k         = ((c*kt + dt)*ph + dy)*pw + dx            (Conv3d weight [D, C, kt, ph, pw])
//
// sm_100a path (f16 / bf16): one CTA per 128-row x BN-column output tile.
//   warps 0-3  gather producers: thread m owns tile row m and, per 64-wide K block,
//              copies its eight 16-byte runs (pw-contiguous image rows) with cp.async
//              straight into the 128B-swizzled K-major A stage; after the copies land
//              it fences them into the async proxy and arrives on the stage barrier.
//              They turn into the epilogue once the accumulator is ready.
//   warp 4     allocates TMEM and issues tcgen05.mma (M=128, N=BN, K=16) from one
//              thread; tcgen05.commit releases each stage and finally the accumulator.
//   warp 5     TMA producer for the weight tile (2-D tiled, 128B swizzle, no multicast).
//   epilogue   tcgen05.ld 32x32b -> + bias -> convert -> store (or scatter into a
//              token cache row, which fuses step 3).
// Every mbarrier wait is bounded in time; on expiry the kernel records an error
// flag, drains its own copies, frees TMEM and returns.
//
// Generic path (f32, or shapes the tensor-core path does not take): a tiled SIMT
// FFMA GEMM over the same gather, f32 accumulation.
#include <cuda.h>

#include <algorithm>
#include <mutex>
#include <string>

#include "common.cuh"
#include "gather_gemm.hpp"
#include "runtime.hpp"
#include "sm100.cuh"
#include "status.hpp"

namespace bjf {
namespace {

using namespace sm100;

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kStagesA = 6;  // gathered tubelet rows (from HBM): deep ring
constexpr int kStagesB = 3;  // weight tiles (L2-resident): shallow ring
constexpr int kMaxBN = 256;
constexpr int kEpilogueWarps = 4;   // warps 0-3: TMEM lane quarters 0-3
constexpr int kProducerWarps = 4;   // warps 4-7: one gathered tile row per thread
constexpr int kMmaWarp = 8;
constexpr int kTmaWarp = 9;
constexpr int kThreads = 32 * 10;
constexpr int kMaxKBlocks = 128;  // K <= 8192
// Waits after a give-up (a role draining its own copies or MMAs) keep the default limit
// whatever bjf_set_bounded_wait chose for the pipeline waits.
constexpr uint64_t kDrainLimitNs = kDefaultWaitLimitNs;

constexpr int kAStageBytes = kBM * kBK * 2;      // 16 KB
constexpr int kBStageBytes = kMaxBN * kBK * 2;   // 32 KB

struct SmemLayout {
  static constexpr int a_off = 0;
  static constexpr int b_off = a_off + kStagesA * kAStageBytes;
  static constexpr int bar_off = b_off + kStagesB * kBStageBytes;
  // full_a[A], empty_a[A], full_b[B], empty_b[B], acc_full[2], acc_empty[2], producers
  static constexpr int misc_off = bar_off + (2 * kStagesA + 2 * kStagesB + 5) * 8;
  // tmem base (4 B), abort flag (4 B), stall barrier (8 B)
  static constexpr int koff_off = misc_off + 16;
  static constexpr int soff_off = koff_off + kMaxKBlocks * 8 * 4;  // stream row offsets
  static constexpr int rowbase_off = soff_off + ((kMaxRowStreams + 1) * 4 + 15) / 16 * 16;
  static constexpr int total = rowbase_off + kBM * 8;
  static constexpr int alloc = total + 1024;  // room to align the base to 1024 B
};
static_assert(SmemLayout::alloc <= 227 * 1024, "single-CTA kernel shared memory");

__device__ __forceinline__ int64_t row_base_offset(const GatherGeometry& g, int4 c, bool& valid) {
  valid = c.x >= 0 && c.x < g.batch && c.y >= 0 && c.y < g.depth && c.z >= 0 && c.z < g.gh &&
          c.w >= 0 && c.w < g.gw;
  if (!valid) return 0;
  return (((int64_t)c.x * g.C * g.Ts + (int64_t)c.y * g.kt) * g.H + (int64_t)c.z * g.ph) * g.W +
         (int64_t)c.w * g.pw;
}

// Loads the stream offsets of an index row source into shared memory (all threads of the
// block) and returns the row count they describe; explicit coords rows return INT32_MAX.
// Stream row offsets soff[0..streams] = exclusive prefix of the per-stream counts (warp 0
// scans 32 streams at a time); returns the row count.  Block-wide.
__device__ __forceinline__ int load_row_offsets(const RowSource& rs, int* soff) {
  if (rs.coords) return 0x7fffffff;
  const int S = rs.streams;
  for (int i = threadIdx.x; i < S; i += blockDim.x) soff[i + 1] = min(max(__ldg(rs.counts + i), 0), rs.index_stride);
  __syncthreads();
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    int carry = 0;
    for (int base = 0; base < S; base += 32) {
      const int i = base + lane;
      int v = i < S ? soff[i + 1] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += y;
      }
      if (i < S) soff[i + 1] = carry + v;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
    if (lane == 0) soff[0] = 0;
  }
  __syncthreads();
  return soff[S];
}

// Coordinates (b, t, r, col) of row m; a token index outside the grid gives t = r = col = -1
// (a zero row, as out-of-range coords).
__device__ __forceinline__ int4 fetch_row(const RowSource& rs, const int* soff, const GatherGeometry& g, int m) {
  if (rs.coords) return __ldg(rs.coords + m);
  int lo = 0, hi = rs.streams;  // soff[lo] <= m < soff[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (soff[mid] <= m) lo = mid; else hi = mid;
  }
  const int idx = __ldg(rs.indices + (int64_t)lo * rs.index_stride + (m - soff[lo]));
  const int tpf = g.gh * g.gw;
  if (idx < 0 || idx >= g.depth * tpf) return make_int4(lo, -1, -1, -1);
  const int t = idx / tpf, rem = idx - t * tpf, r = rem / g.gw;
  return make_int4(lo, t, r, rem - r * g.gw);
}

// The 128 producer threads resolve a tile's 128 rows together: producer thread p resolves
// row p of the tile (resolve_row, issued a tile ahead so its load latency hides behind the
// copies of the current tile) and shares it through rowbase[p], so each row costs one
// dependent load chain per tile rather than eight per thread.  Each thread then picks up
// the eight rows it copies: 32 pw + 4 i + sub.  The producers meet on an mbarrier (`bar`,
// 128 arrivals per phase, `phase` counts this thread's uses) whose waits are bounded like
// every other wait, so a producer that gave up cannot strand the others.  Returns false
// when a wait gave up.
__device__ __forceinline__ int64_t resolve_row(const RowSource& rs, const int* soff, const GatherGeometry& g, int M,
                                               int gm);
__device__ __forceinline__ bool producer_rows(int64_t my_row, int p, int64_t* rowbase, int pw, int sub,
                                              int64_t (&base)[8], uint32_t& valid_mask, uint64_t* bar,
                                              int& phase, volatile int* abort_flag, uint64_t limit_ns);

// Offset of element k of a tubelet row relative to its (b, t*kt, r*ph, col*pw) corner
// (< C*Ts*H*W of one batch element, which the launch checks fits in int32).  In a frame ring
// the tubelet's frames dt = 0, 1 are the ring slots slot0, slot1.
__host__ __device__ __forceinline__ int64_t k_offset(const GatherGeometry& g, int k) {
  int q = k / g.pw;
  int dx = k - q * g.pw;
  int dy = q % g.ph;
  int q2 = q / g.ph;
  int dt = q2 % g.kt;
  int ch = q2 / g.kt;
  const int fr = g.ring ? (dt == 0 ? g.slot0 : g.slot1) : dt;  // a ring clip has depth 1
  return (((int64_t)ch * g.Ts + fr) * g.H + dy) * g.W + dx;
}

// Element offset of row gm in the input, or -1 for a zero row (beyond M or outside the grid).
__device__ __forceinline__ int64_t resolve_row(const RowSource& rs, const int* soff, const GatherGeometry& g, int M,
                                               int gm) {
  if (gm >= M) return -1;
  bool valid = false;
  const int64_t o = row_base_offset(g, fetch_row(rs, soff, g, gm), valid);
  return valid ? o : -1;
}

// A row in two steps, so that its load need not stall the thread that issues it: fetch_row_raw
// issues the load (explicit coords, or the stream and token index; rows beyond M give a
// marker), decode_row turns the loaded value into (b, t, r, col) as fetch_row does, and
// row_offset gives its element offset (-1 for a zero row).
__device__ __forceinline__ int4 fetch_row_raw(const RowSource& rs, const int* soff, int M, int gm) {
  if (gm >= M) return make_int4(-1, -1, -1, -2);
  if (rs.coords) return __ldg(rs.coords + gm);
  int lo = 0, hi = rs.streams;  // soff[lo] <= gm < soff[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (soff[mid] <= gm) lo = mid; else hi = mid;
  }
  return make_int4(lo, __ldg(rs.indices + (int64_t)lo * rs.index_stride + (gm - soff[lo])), 0, 0);
}
__device__ __forceinline__ int4 decode_row(const RowSource& rs, const GatherGeometry& g, int4 raw) {
  if (raw.x == -1 && raw.w == -2) return make_int4(-1, -1, -1, -1);
  if (rs.coords) return raw;
  const int idx = raw.y, tpf = g.gh * g.gw;
  if (idx < 0 || idx >= g.depth * tpf) return make_int4(raw.x, -1, -1, -1);
  const int t = idx / tpf, rem = idx - t * tpf, r = rem / g.gw;
  return make_int4(raw.x, t, r, rem - r * g.gw);
}
__device__ __forceinline__ int64_t row_offset(const GatherGeometry& g, int4 c) {
  bool valid = false;
  const int64_t o = row_base_offset(g, c, valid);
  return valid ? o : -1;
}

__device__ __forceinline__ bool producer_rows(int64_t my_row, int p, int64_t* rowbase, int pw, int sub,
                                              int64_t (&base)[8], uint32_t& valid_mask, uint64_t* bar,
                                              int& phase, volatile int* abort_flag, uint64_t limit_ns) {
  // every producer has read the previous tile's rows
  mbar_arrive(bar);
  if (!mbar_wait_bounded(bar, (uint32_t)(phase++ & 1), abort_flag, limit_ns)) return false;
  rowbase[p] = my_row;
  mbar_arrive(bar);
  if (!mbar_wait_bounded(bar, (uint32_t)(phase++ & 1), abort_flag, limit_ns)) return false;
  valid_mask = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t b = rowbase[32 * pw + 4 * i + sub];
    valid_mask |= (uint32_t)(b >= 0) << i;
    base[i] = b >= 0 ? b : 0;
  }
  return true;
}

// Stores 32 consecutive output columns of one row (ncol of them valid).
template <typename O>
__device__ __forceinline__ void store_chunk(char* dst, const float (&v)[32], int ncol) {
  O* o = reinterpret_cast<O*>(dst);
  if (ncol == 32 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
      float w8[8] = {v[j], v[j + 1], v[j + 2], v[j + 3], v[j + 4], v[j + 5], v[j + 6], v[j + 7]};
      store8<O>(o + j, w8);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < ncol) o[j] = from_f32<O>(v[j]);
  }
}

// Epilogue of one accumulator: this warp's 32 TMEM lanes (tile rows, lane = thread) x bn
// columns from `taddr` -> + bias -> the row's destination (plain [M, D] or its token-cache
// slot, which also marks the slot observed with age 0).  Warp-collective.
// The row's coordinates `c` come from next_row() (fetched before the accumulator wait).
__device__ __forceinline__ int4 next_row(const RowSource& rs, const int* soff, const GatherGeometry& g, int M,
                                         int gm) {
  return gm < M ? fetch_row(rs, soff, g, gm) : make_int4(-1, -1, -1, -1);
}

// Encoder-input epilogue terms for 32 columns starting at col0 (ncol valid): + the row's
// position embedding, then + the modality embedding (src/model.rs:690-703); `mod` holds the
// modality values of these 32 columns, null without one.  Rows without a table row (zero
// rows) stay zero.  Warp-collective (the modality vector is broadcast).
// kVec: 16-byte table loads for full aligned chunks.
template <bool kVec>
__device__ __forceinline__ void add_encoder_embeddings(bool valid, const float* pos_row, const float* mod,
                                                       int col0, int ncol, int lane, float (&v)[32]) {
  if (pos_row) {
    const float* p = pos_row + col0;
    if (kVec && ncol == 32 && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
      // each lane reads its own table row with 16-byte loads
      const float4* p4 = reinterpret_cast<const float4*>(p);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 q = __ldg(p4 + j);
        v[4 * j] = v[4 * j] + q.x;
        v[4 * j + 1] = v[4 * j + 1] + q.y;
        v[4 * j + 2] = v[4 * j + 2] + q.z;
        v[4 * j + 3] = v[4 * j + 3] + q.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < ncol) v[j] = v[j] + __ldg(p + j);
    }
  }
  if (mod) {
    const float ml = lane < ncol ? __ldg(mod + lane) : 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float m = __shfl_sync(0xffffffffu, ml, j);
      if (valid) v[j] = v[j] + m;
    }
  }
}

__device__ __forceinline__ void drain_accumulator(const GatherGeometry& g, const EpilogueArgs& ep, int4 c, int M,
                                                  int gm, int n0, int bn, uint32_t taddr, int lane) {
  const int ce = ep.out_elem_bytes;
  bool valid = false;
  char* dst_row = nullptr;
  const float* pos_row = nullptr;
  if (gm < M) {
    row_base_offset(g, c, valid);
    if (valid && ep.position_table)
      pos_row = ep.position_table + (((int64_t)c.y * g.gh + c.z) * g.gw + c.w) * ep.pos_ld;
    if (ep.mode == kEpiloguePlain) {
      dst_row = static_cast<char*>(ep.out) + (int64_t)gm * ep.ldo * ce;
    } else if (valid) {
      const int64_t idx = ((int64_t)c.y * g.gh + c.z) * g.gw + c.w;
      const int64_t slot = (int64_t)c.x * ep.dense_tokens + idx;
      dst_row = static_cast<char*>(ep.out) + slot * ep.ldo * ce;
      if (n0 == 0) {
        if (ep.observed) ep.observed[slot] = 1.0f;
        if (ep.age) ep.age[slot] = 0.0f;
      }
    }
  }
  for (int c0 = 0; c0 < bn; c0 += 32) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(taddr + (uint32_t)c0, r);
    tmem_ld_wait();
    const int col0 = n0 + c0;
    const int ncol = min(32, min(bn - c0, g.D - col0));  // the same for the whole warp
    if (ncol <= 0) continue;
    // lane j holds bias[col0 + j]; broadcast it to every row of the warp
    const float bl = (ep.bias && lane < ncol) ? __ldg(ep.bias + col0 + lane) : 0.0f;
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float b = __shfl_sync(0xffffffffu, bl, j);
      v[j] = valid ? __uint_as_float(r[j]) + b : 0.0f;
    }
    add_encoder_embeddings<false>(valid, pos_row, ep.modality_embed ? ep.modality_embed + col0 : nullptr, col0, ncol,
                                  lane, v);
    if (!dst_row) continue;
    char* dst = dst_row + (int64_t)col0 * ce;
    if (ep.out_dtype == BJF_DTYPE_F32)
      store_chunk<float>(dst, v, ncol);
    else if (ep.out_dtype == BJF_DTYPE_F16)
      store_chunk<__half>(dst, v, ncol);
    else
      store_chunk<__nv_bfloat16>(dst, v, ncol);
  }
}

// Persistent, warp-specialised gather-GEMM.  grid = min(#SMs, tiles); CTA b takes tiles
// b, b + grid, ... in (m-tile major, n-tile minor) order so concurrently running CTAs share
// their gathered A rows through L2.  Two TMEM accumulators let the epilogue of one tile
// overlap the main loop of the next.
//
// A producers: a 64-wide K block of a tile row is eight 16-byte runs of image rows.  In
// one cp.async instruction a warp copies 4 rows x 8 runs (lane = 8 x row + run), lane pairs
// sharing each 32-byte sector, so an instruction touches 16 sectors rather than 32.  A
// thread owns one run index j (0..7) of eight rows and signals the stage barrier with an
// asynchronous cp.async arrive, so producers never block on their own copies and keep every
// free stage in flight; the MMA thread fences the landed stage into the async proxy before
// issuing on it.
template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    gather_gemm_sm100_kernel(const __grid_constant__ CUtensorMap wmap, const T* __restrict__ video,
                             const RowSource rs, const int32_t* __restrict__ rows_dev,
                             int rows_cap, GatherGeometry g, int bn, EpilogueArgs ep,
                             int* __restrict__ error_flag) {
  extern __shared__ uint8_t smem_dyn[];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  uint8_t* smem = smem_dyn + ((1024 - (smem_u32(smem_dyn) & 1023)) & 1023);
  int* soff = reinterpret_cast<int*>(smem + SmemLayout::soff_off);
  int64_t* rowbase = reinterpret_cast<int64_t*>(smem + SmemLayout::rowbase_off);

  pdl_wait();     // the rows and their count come from the kernels before (plan, selection)
  pdl_trigger();  // the next frame's patch-diff pass may start alongside this GEMM
  int M = rows_cap;
  if (rows_dev) M = min(M, max(0, __ldg(rows_dev)));
  M = min(M, load_row_offsets(rs, soff));
  const int n_tiles = (g.D + bn - 1) / bn;
  const int num_tiles = ((M + kBM - 1) / kBM) * n_tiles;
  if ((int)blockIdx.x >= num_tiles) return;  // uniform early exit before any allocation

  uint64_t* full_a = reinterpret_cast<uint64_t*>(smem + SmemLayout::bar_off);
  uint64_t* empty_a = full_a + kStagesA;
  uint64_t* full_b = empty_a + kStagesA;
  uint64_t* empty_b = full_b + kStagesB;
  uint64_t* acc_full = empty_b + kStagesB;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* prod_bar = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + SmemLayout::misc_off);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + SmemLayout::misc_off + 4);
  uint64_t* stall_bar = reinterpret_cast<uint64_t*>(smem + SmemLayout::misc_off + 8);  // never completes
  int32_t* koff = reinterpret_cast<int32_t*>(smem + SmemLayout::koff_off);

  const int num_kb = g.num_kb;
  if (tid == 0) {
    mbar_init(stall_bar, 1);
    for (int s = 0; s < kStagesA; ++s) {
      mbar_init(&full_a[s], kProducerWarps * 32);
      mbar_init(&empty_a[s], 1);
    }
    for (int s = 0; s < kStagesB; ++s) {
      mbar_init(&full_b[s], 1);
      mbar_init(&empty_b[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpilogueWarps);
    }
    mbar_init(prod_bar, kProducerWarps * 32);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == kTmaWarp && lane == 0) tma_prefetch_desc(&wmap);
  for (int i = tid; i < num_kb * 8; i += kThreads) koff[i] = (int32_t)k_offset(g, i * 8);
  const uint32_t acc_cols = bn <= 32 ? 32 : (bn <= 64 ? 64 : (bn <= 128 ? 128 : 256));
  const uint32_t tmem_cols = 2 * acc_cols;
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const uint32_t a_smem = smem_u32(smem + SmemLayout::a_off);
  const uint32_t b_smem = smem_u32(smem + SmemLayout::b_off);
  bool aborted = false;

  if (warp >= kEpilogueWarps && warp < kEpilogueWarps + kProducerWarps) {
    // ---------------- gather producers (cp.async) ----------------
    const int pw_ = warp - kEpilogueWarps;  // producer warp 0..3: tile rows [32 pw_, 32 pw_ + 32)
    const int j = lane & 7;                 // 16-byte run index within the 128-byte K line
    const int sub = lane >> 3;              // row within a group of 4
    int kbg = 0;  // k blocks issued by this CTA so far (all tiles)
    int prod_phase = 0;
    const int p = tid - kEpilogueWarps * 32;
    int64_t my_row = resolve_row(rs, soff, g, M, ((int)blockIdx.x / n_tiles) * kBM + p);
    for (int tile = blockIdx.x; tile < num_tiles && !aborted; tile += gridDim.x) {
      // this thread's eight rows: m_i = 32 pw_ + 4 i + sub
      int64_t base[8];
      uint32_t dst_off[8];
      uint32_t valid_mask = 0;
      if (!producer_rows(my_row, p, rowbase, pw_, sub, base, valid_mask, prod_bar, prod_phase, abort_flag, g.wait_ns)) {
        aborted = true;
        break;
      }
      const int next = tile + (int)gridDim.x;  // resolved now, used at the next tile
      my_row = next < num_tiles ? resolve_row(rs, soff, g, M, (next / n_tiles) * kBM + p) : -1;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int m = 32 * pw_ + 4 * i + sub;
        dst_off[i] = (uint32_t)((m >> 3) * 1024 + (m & 7) * 128 + ((j ^ (m & 7)) << 4));
      }
      for (int kb = 0; kb < num_kb; ++kb, ++kbg) {
        const int s = kbg % kStagesA;
        const uint32_t par = ((kbg / kStagesA) & 1) ^ 1;
        if (!mbar_wait_bounded(&empty_a[s], par, abort_flag, g.wait_ns)) {
          aborted = true;
          break;
        }
        const uint32_t dst = a_smem + s * kAStageBytes;
        const int64_t ko = koff[kb * 8 + j];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (valid_mask & (1u << i)) cp_async_16(dst + dst_off[i], video + base[i] + ko);
        cp_async_arrive_noinc(&full_a[s]);
      }
    }
    cp_async_wait_all();  // nothing of this thread may still be landing when the CTA exits
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = idesc_f16_f32(g.is_bf16 ? 1u : 0u, kBM, (uint32_t)bn);
      int kbg = 0, it = 0;
      int commits0 = 0;  // tcgen05.commit arrivals on acc_full[0] so far
      bool issued_any = false;
      // Test hook of bjf_set_bounded_wait: a wait that runs out before any MMA is issued, so
      // the give-up path (flag, drains, TMEM release) runs on a normal launch.
      if (g.stall && !mbar_wait_bounded(stall_bar, 0, abort_flag, g.wait_ns)) aborted = true;
      for (int tile = blockIdx.x; tile < num_tiles && !aborted; tile += gridDim.x, ++it) {
        const int buf = it & 1;
        const uint32_t use_par = ((it >> 1) & 1) ^ 1;
        if (!mbar_wait_bounded(&acc_empty[buf], use_par, abort_flag, g.wait_ns)) {
          aborted = true;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)buf * acc_cols;
        for (int kb = 0; kb < num_kb; ++kb, ++kbg) {
          const int sa = kbg % kStagesA, sb = kbg % kStagesB;
          if (!mbar_wait_bounded(&full_a[sa], (kbg / kStagesA) & 1, abort_flag, g.wait_ns) ||
              !mbar_wait_bounded(&full_b[sb], (kbg / kStagesB) & 1, abort_flag, g.wait_ns)) {
            aborted = true;
            break;
          }
          fence_proxy_async_smem();  // the stage's cp.async writes, acquired above, feed the MMA
          tc_fence_after();
          const uint32_t a_base = a_smem + sa * kAStageBytes;
          const uint32_t b_base = b_smem + sb * kBStageBytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            mma_f16_ss(d_tmem, smem_desc_sw128_kmajor(a_base + kk * 32),
                       smem_desc_sw128_kmajor(b_base + kk * 32), idesc, (kb | kk) != 0);
          }
          issued_any = true;
          mma_commit(&empty_a[sa]);
          mma_commit(&empty_b[sb]);
        }
        if (aborted) break;
        mma_commit(&acc_full[buf]);
        commits0 += buf == 0;
      }
      if (aborted && issued_any) {
        // Let the issued MMAs retire before TMEM is freed: one more commit on acc_full[0]
        // completes phase `commits0` once every earlier MMA is done (bounded, abort ignored).
        mma_commit(&acc_full[0]);
        int zero = 0;
        mbar_wait_bounded(&acc_full[0], (uint32_t)(commits0 & 1), &zero, kDrainLimitNs);
      }
    }
  } else if (warp == kTmaWarp) {
    // ---------------- TMA producer (weight) ----------------
    if (lane == 0) {
      int kbg = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !aborted; tile += gridDim.x) {
        const int n0 = (tile % n_tiles) * bn;
        for (int kb = 0; kb < num_kb; ++kb, ++kbg) {
          const int s = kbg % kStagesB;
          const uint32_t par = ((kbg / kStagesB) & 1) ^ 1;
          if (!mbar_wait_bounded(&empty_b[s], par, abort_flag, g.wait_ns)) {
            aborted = true;
            break;
          }
          mbar_arrive_expect_tx(&full_b[s], (uint32_t)(bn * kBK * 2));
          tma_load_2d(b_smem + s * kBStageBytes, &wmap, kb * kBK, n0, &full_b[s]);
        }
      }
      if (aborted) {
        // Wait for the weight tiles still in flight before the CTA's smem goes away.
        int zero = 0;
        for (int k = max(0, kbg - kStagesB); k < kbg; ++k)
          mbar_wait_bounded(&full_b[k % kStagesB], (k / kStagesB) & 1, &zero, kDrainLimitNs);
      }
    }
  } else {
    // ---------------- epilogue (warps 0-3) ----------------
    const int m = tid;  // TMEM lane = tile row
    int it = 0;
    int4 c = next_row(rs, soff, g, M, ((int)blockIdx.x / n_tiles) * kBM + m);
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
      const int buf = it & 1;
      const uint32_t par = (it >> 1) & 1;
      bool ok = mbar_wait_bounded(&acc_full[buf], par, abort_flag, g.wait_ns);
      if (__any_sync(0xffffffffu, !ok)) {  // tcgen05.ld is warp-collective: decide per warp
        aborted = true;
        break;
      }
      tc_fence_after();
      const int n0 = (tile % n_tiles) * bn;
      const int gm = (tile / n_tiles) * kBM + m;
      drain_accumulator(g, ep, c, M, gm, n0, bn, tmem_base + (uint32_t)buf * acc_cols + ((uint32_t)(warp * 32) << 16),
                        lane);
      // This warp has finished reading accumulator `buf`: hand it back to the MMA warp.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      const int next = tile + (int)gridDim.x;
      if (next < num_tiles) c = next_row(rs, soff, g, M, (next / n_tiles) * kBM + m);
    }
  }

  if (aborted) {
    *abort_flag = 1;
    atomicExch(error_flag, 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, tmem_cols);
  }
}

// ---------------------------------------------------------------------------
// CTA-pair path: 256 x BN tiles on two SMs (tcgen05 cta_group::2)
// ---------------------------------------------------------------------------
// A cluster of two CTAs computes a 256-row x BN-column tile: each CTA gathers its own 128
// rows of A and loads half of the BN weight rows (B) by TMA into the same shared-memory
// offsets, and the even CTA issues tcgen05.mma.cta_group::2 (M = 256) that reads both CTAs'
// operands and writes 128 rows of D into each CTA's TMEM.  Per SM this halves the weight
// traffic of the 128 x BN tile of the single-CTA kernel for the same tensor work.  BN = 256
// whenever D > 256 (D = 1408 runs five full column tiles and a half-empty sixth): A is gathered
// once per 256 output columns, and the gather -- bound by its request rate, each 32-byte patch
// row of a tubelet in its own cache line -- is what limits the main loop.  Two TMEM
// accumulators of 256 columns let a tile's epilogue overlap the next tile's MMAs.
//
// (Tiles of 256 x 512 with one accumulator filling TMEM gather A half as often and ran the
// main loop at about 1.3 PFLOP/s, but the epilogue then stalls the tensor pipe for each tile,
// and the whole was slower than overlapped 256-column tiles.)
//
// Stage handshake: a stage (16 KB of gathered rows + BN/2 x 64 weight rows per CTA) is full in
// a CTA when its 128 producer threads' cp.async arrivals and its TMA bytes have landed.
// cp.async and TMA can only signal barriers of their own CTA, so lanes of the odd CTA's MMA
// warp relay, one lane per stage: a lane waits for its stage's local full barrier, fences
// the stage into the async proxy and arrives (relaxed, cluster scope) on the even CTA's
// peer_full barrier.  The MMA thread waits for both CTAs' stages, issues, and
// tcgen05.commit multicasts the stage release (empty) and the accumulator-ready signal
// (acc_full) to both CTAs.  Both CTAs' epilogue warps hand the accumulator back on the even
// CTA's acc_empty barrier.
//
// Epilogue: each epilogue warp converts its 32 accumulator rows 64 output bytes per row at a
// time into a shared-memory staging tile and writes the staged rows back with 16-byte stores,
// four lanes per row (drain_accumulator_rows).
constexpr int kPairStages = 5;
constexpr int kBHalfStageBytes = (kMaxBN / 2) * kBK * 2;  // 16 KB: 128 weight rows x 64
constexpr int kEpiRowBytes = 64;                          // output bytes per row per staged chunk
constexpr int kEpiRowPitch = kEpiRowBytes + 16;           // rows a quarter-warp writes fall in distinct banks
constexpr int kEpiWarpBytes = 32 * kEpiRowPitch + 32 * 8; // one warp's staging tile + its 32 row addresses
static_assert(kPairStages <= 32, "one relay lane per stage");

template <bool kEmbed>
struct PairSmemLayout {
  // per tile: bias (and, kEmbed, modality) of its columns, two tiles' worth
  static constexpr int kColBufFloats = (kEmbed ? 2 : 1) * kMaxBN;
  static constexpr int a_off = 0;
  static constexpr int b_off = a_off + kPairStages * kAStageBytes;
  static constexpr int epi_off = b_off + kPairStages * kBHalfStageBytes;     // epilogue warps' staging
  static constexpr int pepi_off = epi_off + kEpilogueWarps * kEpiWarpBytes;  // producer warps' staging
  static constexpr int col_off = pepi_off + kProducerWarps * kEpiWarpBytes;
  static constexpr int bar_off = col_off + 2 * kColBufFloats * 4;
  // full[S], peer_full[S], empty[S], acc_full[2], acc_empty[2], producers, col_ready[2]
  static constexpr int misc_off = bar_off + (3 * kPairStages + 7) * 8;
  // tmem base (4 B), abort flag (4 B)
  static constexpr int rowbase_off = misc_off + 16;
  static constexpr int koff_off = rowbase_off + kBM * 8;
  // then the K-offset table (num_kb * 8 ints) and the stream row offsets (streams + 1 ints),
  // sized at launch; + 1 KB to align the base to 1024 bytes
  static constexpr size_t bytes(int num_kb, int streams) {
    return (size_t)koff_off + (size_t)num_kb * 32 + ((size_t)streams + 1) * 4 + 1024;
  }
  // more than half of an SM's 228 KB: one CTA per SM whatever the launch's stream count
  static_assert(koff_off > 114 * 1024, "pair kernel residency");
};
static_assert(PairSmemLayout<true>::bytes(kMaxKBlocks, kMaxRowStreams) <= 227 * 1024, "pair kernel smem");

// Converts 16 values to the output type and stores them at `dst` (shared memory, 16-byte
// aligned): packed two-element conversions, 16-byte stores.
template <typename O>
__device__ __forceinline__ void pack16(uint8_t* dst, const float (&v)[16]);
template <>
__device__ __forceinline__ void pack16<float>(uint8_t* dst, const float (&v)[16]) {
  float4* d = reinterpret_cast<float4*>(dst);
#pragma unroll
  for (int q = 0; q < 4; ++q) d[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
}
template <>
__device__ __forceinline__ void pack16<__half>(uint8_t* dst, const float (&v)[16]) {
  uint32_t w[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const __half2 h = __floats2half2_rn(v[2 * q], v[2 * q + 1]);
    w[q] = *reinterpret_cast<const uint32_t*>(&h);
  }
  reinterpret_cast<uint4*>(dst)[0] = make_uint4(w[0], w[1], w[2], w[3]);
  reinterpret_cast<uint4*>(dst)[1] = make_uint4(w[4], w[5], w[6], w[7]);
}
template <>
__device__ __forceinline__ void pack16<__nv_bfloat16>(uint8_t* dst, const float (&v)[16]) {
  uint32_t w[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * q], v[2 * q + 1]);
    w[q] = *reinterpret_cast<const uint32_t*>(&h);
  }
  reinterpret_cast<uint4*>(dst)[0] = make_uint4(w[0], w[1], w[2], w[3]);
  reinterpret_cast<uint4*>(dst)[1] = make_uint4(w[4], w[5], w[6], w[7]);
}

// Epilogue of one accumulator through a per-warp staging tile and line-wide stores: this
// warp's 32 TMEM lanes (tile rows, lane = thread) x columns [c_begin, c_end) from `taddr` ->
// + bias (-> + embeddings) -> converted -> each row's destination (plain [M, D], or its
// token-cache slot, which also marks the slot observed with age 0).
//
// Per chunk of 64 output bytes per row (32 columns of 16-bit output, 16 of f32) each lane
// stages its own row 16 columns at a time -- one tcgen05.ld of 16 columns, the bias (and
// modality) as broadcast 16-byte shared-memory loads, packed conversions, 16-byte shared
// stores -- and the warp then writes the 32 staged rows back eight at a time, four lanes x 16
// bytes per row (the row addresses read from shared memory).  The per-row work is short,
// independent instruction runs: the warp issues in order under an 80-register budget, and a
// column loop of dependent shuffle -> add pairs (one shuffle per column to broadcast the bias)
// ran at one instruction per latency.
// bias_s / mod_s: the bias and modality values of accumulator columns [0, c_end) (shared
// memory, 16-byte aligned, staged ahead by the epilogue warps; mod_s null without a modality
// vector).  `stage` is this warp's staging tile: 32 rows x kEpiRowPitch bytes, then 32 row
// addresses.  c_begin is a multiple of the chunk width.  Warp-collective.
template <bool kEmbed>
__device__ __forceinline__ void drain_accumulator_rows(const GatherGeometry& g, const EpilogueArgs& ep, int4 c,
                                                       int M, int gm, int n0, int c_begin, int c_end, uint32_t taddr,
                                                       int lane, uint8_t* stage, const float* bias_s,
                                                       const float* mod_s, char* out_base) {
  const int ce = ep.out_elem_bytes;
  bool valid = false;
  char* dst_row = nullptr;
  const float* pos_row = nullptr;
  if (gm < M) {
    row_base_offset(g, c, valid);
    if (valid && ep.position_table)
      pos_row = ep.position_table + (((int64_t)c.y * g.gh + c.z) * g.gw + c.w) * ep.pos_ld;
    if (ep.mode == kEpiloguePlain) {
      dst_row = out_base + (int64_t)gm * ep.ldo * ce;
    } else if (valid) {
      const int64_t idx = ((int64_t)c.y * g.gh + c.z) * g.gw + c.w;
      const int64_t slot = (int64_t)c.x * ep.dense_tokens + idx;
      dst_row = out_base + slot * ep.ldo * ce;
      if (n0 == 0) {
        if (ep.observed) ep.observed[slot] = 1.0f;
        if (ep.age) ep.age[slot] = 0.0f;
      }
    }
  }
  // 16-byte stores need 16-byte aligned rows (output base and row pitch; column offsets of a
  // chunk are multiples of 32 bytes)
  const bool vec = ((reinterpret_cast<uintptr_t>(out_base) | (uintptr_t)(ep.ldo * ce)) & 15) == 0;
  const int cpc = kEpiRowBytes / ce;  // columns per chunk
  char** rowptr = reinterpret_cast<char**>(stage + 32 * kEpiRowPitch);
  __syncwarp();  // the previous drain's write-back has read the row addresses
  rowptr[lane] = dst_row;
  uint8_t* srow = stage + lane * kEpiRowPitch;
  constexpr int kSegs = kEpiRowBytes / 16;  // 16-byte segments of a staged row
  const int seg = lane % kSegs;             // this lane's segment of a row in the write-back
  // Encoder input: the row's position values of the next 16 columns are loaded one subchunk
  // ahead, so their L2 latency overlaps this subchunk's TMEM load, conversion and write-back.
  const int pos_lim = min(c_end, g.D - n0);  // columns of this drain inside the row
  float pnext[16];
  auto load_pos = [&](int col) {  // the 16 values from column col (zeros past the row's end)
    if (!kEmbed || !pos_row || col >= pos_lim) return;
    const float* p = pos_row + n0 + col;
    if (col + 16 <= pos_lim && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(p) + k);
        pnext[4 * k] = t.x;
        pnext[4 * k + 1] = t.y;
        pnext[4 * k + 2] = t.z;
        pnext[4 * k + 3] = t.w;
      }
    } else {
#pragma unroll
      for (int k = 0; k < 16; ++k) pnext[k] = col + k < pos_lim ? __ldg(p + k) : 0.0f;
    }
  };
  if (kEmbed) load_pos(c_begin);
  for (int c0 = c_begin; c0 < c_end; c0 += cpc) {
    const int col0 = n0 + c0;
    const int ncol = min(cpc, min(c_end - c0, g.D - col0));  // the same for the whole warp
    if (ncol <= 0) break;
    __syncwarp();  // the previous chunk's staged rows have been written out
    for (int q = 0; q * 16 < ncol; ++q) {
      float pcur[16];
      if (kEmbed) {
#pragma unroll
        for (int k = 0; k < 16; ++k) pcur[k] = pnext[k];
        load_pos(c0 + 16 * q + 16);
      }
      uint32_t r[16];
      tmem_ld_32x32b_x16(taddr + (uint32_t)(c0 + 16 * q), r);
      tmem_ld_wait();
      const float4* b4 = reinterpret_cast<const float4*>(bias_s + c0 + 16 * q);  // same address in every lane
      float v[16];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float4 b = b4[k];
        v[4 * k] = valid ? __uint_as_float(r[4 * k]) + b.x : 0.0f;
        v[4 * k + 1] = valid ? __uint_as_float(r[4 * k + 1]) + b.y : 0.0f;
        v[4 * k + 2] = valid ? __uint_as_float(r[4 * k + 2]) + b.z : 0.0f;
        v[4 * k + 3] = valid ? __uint_as_float(r[4 * k + 3]) + b.w : 0.0f;
      }
      if (kEmbed) {
        if (pos_row) {  // the row's position embedding (this lane's own table row)
#pragma unroll
          for (int k = 0; k < 16; ++k) v[k] = v[k] + pcur[k];
        }
        if (mod_s && valid) {  // then the modality embedding (broadcast, like the bias)
          const float4* m4 = reinterpret_cast<const float4*>(mod_s + c0 + 16 * q);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float4 mm = m4[k];
            v[4 * k] = v[4 * k] + mm.x;
            v[4 * k + 1] = v[4 * k + 1] + mm.y;
            v[4 * k + 2] = v[4 * k + 2] + mm.z;
            v[4 * k + 3] = v[4 * k + 3] + mm.w;
          }
        }
      }
      uint8_t* d = srow + 16 * q * ce;
      if (ep.out_dtype == BJF_DTYPE_F32)
        pack16<float>(d, v);
      else if (ep.out_dtype == BJF_DTYPE_F16)
        pack16<__half>(d, v);
      else
        pack16<__nv_bfloat16>(d, v);
    }
    __syncwarp();  // every row of the chunk is staged
    const int left = ncol * ce - seg * 16;  // bytes of this lane's segment that lie inside the chunk
    if (left > 0) {
#pragma unroll 4
      for (int r0 = 0; r0 < 32; r0 += 32 / kSegs) {
        const int rr = r0 + lane / kSegs;
        char* d = rowptr[rr];  // the same address in the lanes of a row
        if (!d) continue;
        d += (int64_t)col0 * ce + seg * 16;
        const uint8_t* sp = stage + rr * kEpiRowPitch + seg * 16;
        if (vec && left >= 16) {
          *reinterpret_cast<uint4*>(d) = *reinterpret_cast<const uint4*>(sp);
        } else {
          for (int k = 0; k < min(left, 16); ++k) d[k] = static_cast<char>(sp[k]);
        }
      }
    }
  }
}

// Relaxed arrive on another CTA's mbarrier: the stage it announces has already landed in
// shared memory and been fenced into the async proxy by the relaying thread.
__device__ __forceinline__ void mbar_arrive_remote_relaxed(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// At most 80 registers per thread: with three of the ten warps on one SM sub-partition that
// leaves room beside each CTA for two blocks of the next frame's patch-diff pass (which
// programmatic dependent launch starts while this kernel runs).  kEmbed: the instantiation for
// the encoder-input epilogue, whose position-table loads need more registers (it never runs
// beside the patch-diff pass, so it may take them).
template <typename T, bool kEmbed>
__global__ void __maxnreg__(kEmbed ? 128 : 80)
    gather_gemm_sm100_pair_kernel(const __grid_constant__ CUtensorMap wmap, const T* __restrict__ video,
                                  const RowSource rs, const int32_t* __restrict__ rows_dev,
                                  int rows_cap, GatherGeometry g, int bn, EpilogueArgs ep,
                                  int* __restrict__ error_flag) {
  using L = PairSmemLayout<kEmbed>;
  extern __shared__ uint8_t smem_dyn[];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  // both CTAs use the same dynamic shared memory base, so offsets agree across the pair
  uint8_t* smem = smem_dyn + ((1024 - (smem_u32(smem_dyn) & 1023)) & 1023);
  int64_t* rowbase = reinterpret_cast<int64_t*>(smem + L::rowbase_off);
  int32_t* koff = reinterpret_cast<int32_t*>(smem + L::koff_off);
  const int num_kb = g.num_kb;
  int* soff = koff + num_kb * 8;  // stream row offsets, after the K-offset table

  const uint32_t rank = cluster_ctarank();  // 0: issues the MMAs
  const int cluster = (int)(blockIdx.x >> 1);
  const int nclusters = (int)(gridDim.x >> 1);
  const int n_tiles = (g.D + bn - 1) / bn;
  // a work unit is a 256 x bn tile, or with split K one of its ks K ranges of kbs blocks
  const int ks = max(g.ksplit, 1), kbs = (num_kb + ks - 1) / ks;
  auto unit_row = [&](int u) { return (u / ks) / n_tiles; };
  auto unit_col = [&](int u) { return (u / ks) % n_tiles; };
  auto unit_kb0 = [&](int u) { return (u % ks) * kbs; };
  auto unit_kb1 = [&](int u) { return min(num_kb, (u % ks + 1) * kbs); };
  auto unit_out = [&](int u) { return static_cast<char*>(ep.out) + (int64_t)(u % ks) * ep.split_stride; };
  const int half = bn >> 1;  // weight rows per CTA
  // On the CTA's last tile the producer warps, idle by then, drain accumulator columns
  // [split, bn) while the epilogue warps drain [0, split): a chunk-aligned half.  They wait for
  // the accumulator's phase by parity, unambiguous only if the MMAs are at most one phase of
  // that buffer behind, which the ring guarantees from two K stages per tile on (with one, the
  // epilogue warps drain it all).
  const int epi_chunk_cols = kEpiRowBytes / ep.out_elem_bytes;
  const int split = num_kb - (ks - 1) * kbs >= 2 ? (bn / 2) / epi_chunk_cols * epi_chunk_cols : 0;

  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::bar_off);
  uint64_t* peer_full = full + kPairStages;
  uint64_t* empty = peer_full + kPairStages;
  uint64_t* acc_full = empty + kPairStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* prod_bar = acc_empty + 2;
  uint64_t* col_ready = prod_bar + 1;  // [2]: a tile's column buffer is staged
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::misc_off);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::misc_off + 4);
  float* colbuf = reinterpret_cast<float*>(smem + L::col_off);  // [2][kColBufFloats]

  if (tid == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&full[s], kProducerWarps * 32 + 1);  // 128 cp.async arrivals + the TMA thread
      mbar_init(&peer_full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * kEpilogueWarps);  // epilogue warps of both CTAs
    }
    mbar_init(prod_bar, kProducerWarps * 32);
    for (int b = 0; b < 2; ++b) mbar_init(&col_ready[b], kEpilogueWarps * 32);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == kTmaWarp && lane == 0) tma_prefetch_desc(&wmap);
  for (int i = tid; i < num_kb * 8; i += kThreads) koff[i] = (int32_t)k_offset(g, i * 8);
  const uint32_t acc_cols = bn <= 32 ? 32 : (bn <= 64 ? 64 : (bn <= 128 ? 128 : 256));
  const uint32_t tmem_cols = 2 * acc_cols;
  if (warp == kMmaWarp) {
    tmem_alloc_pair(tmem_slot, tmem_cols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised and TMEM allocated before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // Everything above depends only on the geometry, so it overlaps the kernel before (the
  // selection); the rows and their count come from it.  The trigger comes after the wait: the
  // next frame's patch-diff pass rewrites the scores the selection reads.
  pdl_wait();
  pdl_trigger();  // the next frame's patch-diff pass may start alongside this GEMM
  int M = rows_cap;
  if (rows_dev) M = min(M, max(0, __ldg(rows_dev)));
  M = min(M, load_row_offsets(rs, soff));
  const int num_tiles = ((M + 2 * kBM - 1) / (2 * kBM)) * n_tiles * ks;  // units of 256-row pair tiles
  if (cluster >= num_tiles) {  // the same for both CTAs of the pair
    tc_fence_before();
    cluster_sync();
    if (warp == kMmaWarp) {
      tc_fence_after();
      tmem_dealloc_pair(tmem_base, tmem_cols);
    }
    return;
  }
  const int my_tiles = (num_tiles - cluster + nclusters - 1) / nclusters;

  const uint32_t a_smem = smem_u32(smem + L::a_off);
  const uint32_t b_smem = smem_u32(smem + L::b_off);
  bool aborted = false;
  auto acc_tmem = [&](int it) { return tmem_base + (uint32_t)(it & 1) * acc_cols; };
  // The bias (and modality) values of the `it`-th tile's columns, staged in shared memory by the
  // epilogue warps a tile ahead, buffer it & 1, published on col_ready[it & 1].  A global load
  // issued in the drain itself would wait behind the producers' in-flight gathers on the
  // critical path.  A buffer is rewritten for tile it + 2 only after every epilogue warp
  // drained tile it (the MMAs of tile it + 2 need that accumulator back), so the reuse needs no
  // further synchronisation.
  auto col_bias = [&](int it) { return colbuf + (it & 1) * L::kColBufFloats; };
  auto col_mod = [&](int it) { return kEmbed && ep.modality_embed ? col_bias(it) + kMaxBN : nullptr; };

  if (warp >= kEpilogueWarps && warp < kEpilogueWarps + kProducerWarps) {
    // ---------------- gather producers (cp.async), both CTAs ----------------
    const int pw_ = warp - kEpilogueWarps;  // = this warp's TMEM lane quarter (warp % 4)
    const int j = lane & 7;
    const int sub = lane >> 3;
    int kbg = 0;
    int prod_phase = 0;
    const int p = tid - kEpilogueWarps * 32;  // this thread's tile row: 32 pw_ + lane
    const int row_in_pair = (int)rank * kBM + p;
    // A tile's row is loaded (index or coords) when the tile before starts and decoded when it
    // ends, so the load's latency never stalls the in-order issue of the copies.
    int4 raw = fetch_row_raw(rs, soff, M, unit_row(cluster) * (2 * kBM) + row_in_pair);
    int4 c_this = decode_row(rs, g, raw);
    int64_t my_row = row_offset(g, c_this);
    for (int tile = cluster; tile < num_tiles && !aborted; tile += nclusters) {
      int64_t base[8];
      uint32_t dst_off[8];
      uint32_t valid_mask = 0;
      const bool rows_ok = producer_rows(my_row, p, rowbase, pw_, sub, base, valid_mask, prod_bar, prod_phase,
                                         abort_flag, g.wait_ns);
      if (__any_sync(0xffffffffu, !rows_ok)) {
        aborted = true;
        break;
      }
      const int next = tile + nclusters;
      if (next < num_tiles) raw = fetch_row_raw(rs, soff, M, unit_row(next) * (2 * kBM) + row_in_pair);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int m = 32 * pw_ + 4 * i + sub;
        dst_off[i] = (uint32_t)((m >> 3) * 1024 + (m & 7) * 128 + ((j ^ (m & 7)) << 4));
      }
      for (int kb = unit_kb0(tile); kb < unit_kb1(tile); ++kb, ++kbg) {
        const int s = kbg % kPairStages;
        const uint32_t par = ((kbg / kPairStages) & 1) ^ 1;
        const bool ok = mbar_wait_bounded(&empty[s], par, abort_flag, g.wait_ns);
        if (__any_sync(0xffffffffu, !ok)) {
          aborted = true;
          break;
        }
        const uint32_t dst = a_smem + s * kAStageBytes;
        const int64_t ko = koff[kb * 8 + j];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (valid_mask & (1u << i)) cp_async_16(dst + dst_off[i], video + base[i] + ko);
        cp_async_arrive_noinc(&full[s]);
      }
      if (next < num_tiles) {
        c_this = decode_row(rs, g, raw);
        my_row = row_offset(g, c_this);
      }
    }
    cp_async_wait_all();
    // Help drain the last accumulator, columns [split, bn), through this warp's own staging
    // area.  Warp-uniform (the drain is warp-collective).
    if (!aborted && split > 0 && my_tiles > 0) {
      const int it_last = my_tiles - 1;
      const bool ok = mbar_wait_bounded(&acc_full[it_last & 1], (uint32_t)((it_last >> 1) & 1), abort_flag,
                                        g.wait_ns) &&
                      mbar_wait_bounded(&col_ready[it_last & 1], (uint32_t)((it_last >> 1) & 1), abort_flag,
                                        g.wait_ns);
      if (__any_sync(0xffffffffu, !ok)) {
        aborted = true;
      } else {
        tc_fence_after();
        const int tile = cluster + it_last * nclusters;
        uint8_t* pstage = smem + L::pepi_off + pw_ * kEpiWarpBytes;
        drain_accumulator_rows<kEmbed>(g, ep, c_this, M, unit_row(tile) * (2 * kBM) + row_in_pair,
                                       unit_col(tile) * bn, split, bn,
                                       acc_tmem(it_last) + ((uint32_t)(pw_ * 32) << 16), lane, pstage,
                                       col_bias(it_last), col_mod(it_last), unit_out(tile));
        tc_fence_before();
      }
    }
  } else if (warp == kMmaWarp) {
    if (rank == 0 && lane == 0) {
      // ---------------- MMA issuer (even CTA) ----------------
      const uint32_t idesc = idesc_f16_f32(g.is_bf16 ? 1u : 0u, 2 * kBM, (uint32_t)bn);
      int kbg = 0, it = 0;
      int commits0 = 0;
      bool issued_any = false;
      for (int tile = cluster; tile < num_tiles && !aborted; tile += nclusters, ++it) {
        const int buf = it & 1;
        const uint32_t use_par = ((it >> 1) & 1) ^ 1;
        if (!mbar_wait_bounded_cluster(&acc_empty[buf], use_par, abort_flag, g.wait_ns)) {
          aborted = true;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = acc_tmem(it);
        const int kb0 = unit_kb0(tile);
        for (int kb = kb0; kb < unit_kb1(tile); ++kb, ++kbg) {
          const int s = kbg % kPairStages;
          const uint32_t par = (kbg / kPairStages) & 1;
          if (!mbar_wait_bounded(&full[s], par, abort_flag, g.wait_ns) ||
              !mbar_wait_bounded_cluster(&peer_full[s], par, abort_flag, g.wait_ns)) {
            aborted = true;
            break;
          }
          fence_proxy_async_smem();  // this CTA's landed cp.async writes feed the MMA
          tc_fence_after();
          const uint32_t a_base = a_smem + s * kAStageBytes;
          const uint32_t b_base = b_smem + s * kBHalfStageBytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            mma_f16_ss_pair(d_tmem, smem_desc_sw128_kmajor(a_base + kk * 32),
                            smem_desc_sw128_kmajor(b_base + kk * 32), idesc, kb != kb0 || kk != 0);
          }
          issued_any = true;
          mma_commit_pair(&empty[s], 0x3);
        }
        if (aborted) break;
        mma_commit_pair(&acc_full[buf], 0x3);
        commits0 += buf == 0;
      }
      if (aborted && issued_any) {
        // the issued MMAs read both CTAs' shared memory and write both TMEMs: let them retire
        // (a commit to this CTA only; bounded, abort ignored)
        mma_commit_pair(&acc_full[0], 0x1);
        int zero = 0;
        mbar_wait_bounded(&acc_full[0], (uint32_t)(commits0 & 1), &zero, kDrainLimitNs);
      }
    } else if (rank == 1 && lane < kPairStages) {
      // ---------------- stage relay (odd CTA): lane s relays stage s ----------------
      const int s = lane;
      const uint32_t remote = cluster_map(smem_u32(&peer_full[s]), 0);
      int total_kb = 0;  // K blocks of this cluster's units
      for (int u = cluster; u < num_tiles; u += nclusters) total_kb += unit_kb1(u) - unit_kb0(u);
      for (int kbg = s; kbg < total_kb; kbg += kPairStages) {
        if (!mbar_wait_bounded(&full[s], (kbg / kPairStages) & 1, abort_flag, g.wait_ns)) {
          aborted = true;
          break;
        }
        fence_proxy_async_smem();  // this CTA's landed stage feeds the peer's MMA
        mbar_arrive_remote_relaxed(remote);
      }
    }
  } else if (warp == kTmaWarp) {
    // ---------------- TMA producer (this CTA's half of the weight rows) ----------------
    if (lane == 0) {
      int kbg = 0;
      for (int tile = cluster; tile < num_tiles && !aborted; tile += nclusters) {
        const int n0 = unit_col(tile) * bn + (int)rank * half;
        for (int kb = unit_kb0(tile); kb < unit_kb1(tile); ++kb, ++kbg) {
          const int s = kbg % kPairStages;
          const uint32_t par = ((kbg / kPairStages) & 1) ^ 1;
          if (!mbar_wait_bounded(&empty[s], par, abort_flag, g.wait_ns)) {
            aborted = true;
            break;
          }
          mbar_arrive_expect_tx(&full[s], (uint32_t)(half * kBK * 2));
          tma_load_2d(b_smem + s * kBHalfStageBytes, &wmap, kb * kBK, n0, &full[s]);
        }
      }
      // Every stage release is a multicast from the even CTA's MMA thread: wait until the
      // last one of each stage has landed here before this CTA's shared memory goes away.
      int zero = 0;
      const uint64_t limit = aborted ? 1000000ull : kDrainLimitNs;
      for (int k = max(0, kbg - kPairStages); k < kbg; ++k)
        mbar_wait_bounded(&empty[k % kPairStages], (k / kPairStages) & 1, &zero, limit);
    }
  } else {
    // ---------------- epilogue (warps 0-3, both CTAs) ----------------
    const int m = tid;
    const uint32_t remote_acc_empty = cluster_map(smem_u32(&acc_empty[0]), 0);
    uint8_t* stage = smem + L::epi_off + warp * kEpiWarpBytes;
    const uint32_t lanes = (uint32_t)(warp * 32) << 16;
    int it = 0;
    int4 c = next_row(rs, soff, g, M, unit_row(cluster) * (2 * kBM) + (int)rank * kBM + m);
    auto stage_columns = [&](int it_) {
      const int n0_ = unit_col(cluster + it_ * nclusters) * bn;
      float* dst = col_bias(it_);
      for (int jj = tid; jj < bn; jj += kEpilogueWarps * 32) {
        const int col = n0_ + jj;
        dst[jj] = (ep.bias && col < g.D) ? __ldg(ep.bias + col) : 0.0f;
        if (kEmbed) dst[kMaxBN + jj] = (ep.modality_embed && col < g.D) ? __ldg(ep.modality_embed + col) : 0.0f;
      }
      mbar_arrive(&col_ready[it_ & 1]);
    };
    stage_columns(0);
    for (int tile = cluster; tile < num_tiles; tile += nclusters, ++it) {
      const int buf = it & 1;
      const bool ok = mbar_wait_bounded(&acc_full[buf], (uint32_t)((it >> 1) & 1), abort_flag, g.wait_ns) &&
                      mbar_wait_bounded(&col_ready[buf], (uint32_t)((it >> 1) & 1), abort_flag, g.wait_ns);
      if (__any_sync(0xffffffffu, !ok)) {
        aborted = true;
        break;
      }
      tc_fence_after();
      const int n0 = unit_col(tile) * bn;
      const int gm = unit_row(tile) * (2 * kBM) + (int)rank * kBM + m;
      const bool last = tile + nclusters >= num_tiles;
      drain_accumulator_rows<kEmbed>(g, ep, c, M, gm, n0, 0, last && split > 0 ? split : bn, acc_tmem(it) + lanes,
                                     lane, stage, col_bias(it), col_mod(it), unit_out(tile));
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0)
          mbar_arrive(&acc_empty[buf]);
        else
          mbar_arrive_remote(remote_acc_empty + (uint32_t)buf * 8);
      }
      const int next = tile + nclusters;
      if (next < num_tiles) {
        c = next_row(rs, soff, g, M, unit_row(next) * (2 * kBM) + (int)rank * kBM + m);
        stage_columns(it + 1);
      }
    }
  }

  if (aborted) {
    *abort_flag = 1;
    atomicExch(error_flag, 1);
  }
  tc_fence_before();
  cluster_sync();  // no CTA leaves while its peer may still touch its barriers, smem or TMEM
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, tmem_cols);
  }
}

// ---------------------------------------------------------------------------
// SIMT path
// ---------------------------------------------------------------------------
constexpr int kSBM = 64, kSBN = 64, kSBK = 32, kSThreads = 256;

template <typename TIn, typename TW>
__global__ void __launch_bounds__(kSThreads)
    gather_gemm_simt_kernel(const TIn* __restrict__ video, const RowSource rs,
                            const int32_t* __restrict__ rows_dev, int rows_cap, GatherGeometry g,
                            const TW* __restrict__ weight, EpilogueArgs ep) {
  __shared__ int soff[kMaxRowStreams + 1];
  __shared__ float As[kSBK][kSBM + 4];
  __shared__ float Ws[kSBK][kSBN + 4];
  __shared__ int64_t row_base[kSBM];
  __shared__ int row_valid[kSBM];
  __shared__ int4 row_c[kSBM];
  __shared__ int64_t koffs[kSBK];

  pdl_wait();
  pdl_trigger();
  int M = rows_cap;
  if (rows_dev) M = min(M, max(0, __ldg(rows_dev)));
  M = min(M, load_row_offsets(rs, soff));
  const int m0 = blockIdx.y * kSBM;
  if (m0 >= M) return;
  const int n0 = blockIdx.x * kSBN;
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;

  if (tid < kSBM) {
    const int gm = m0 + tid;
    bool valid = false;
    int64_t base = 0;
    int4 c = make_int4(-1, -1, -1, -1);
    if (gm < M) {
      c = fetch_row(rs, soff, g, gm);
      base = row_base_offset(g, c, valid);
    }
    row_base[tid] = base;
    row_valid[tid] = valid;
    row_c[tid] = c;
  }
  float acc[4][4] = {};
  for (int k0 = 0; k0 < g.K; k0 += kSBK) {
    __syncthreads();
    if (tid < kSBK) koffs[tid] = (k0 + tid < g.K) ? k_offset(g, k0 + tid) : 0;
    __syncthreads();
    for (int e = tid; e < kSBM * kSBK; e += kSThreads) {
      const int m = e / kSBK, k = e % kSBK;
      float v = 0.0f;
      if (row_valid[m] && k0 + k < g.K) v = to_f32<TIn>(video[row_base[m] + koffs[k]]);
      As[k][m] = v;
    }
    for (int e = tid; e < kSBN * kSBK; e += kSThreads) {
      const int n = e / kSBK, k = e % kSBK;
      float v = 0.0f;
      if (n0 + n < g.D && k0 + k < g.K) v = to_f32<TW>(weight[(int64_t)(n0 + n) * g.K + k0 + k]);
      Ws[k][n] = v;
    }
    __syncthreads();
#pragma unroll 8
    for (int k = 0; k < kSBK; ++k) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[k][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Ws[k][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
  }
  const int ce = ep.out_elem_bytes;
  for (int i = 0; i < 4; ++i) {
    const int m = ty * 4 + i;
    const int gm = m0 + m;
    if (gm >= M) continue;
    const bool valid = row_valid[m];
    char* dst_row = nullptr;
    if (ep.mode == kEpiloguePlain) {
      dst_row = static_cast<char*>(ep.out) + (int64_t)gm * ep.ldo * ce;
    } else if (valid) {
      const int4 c = row_c[m];
      const int64_t slot = (int64_t)c.x * ep.dense_tokens + ((int64_t)c.y * g.gh + c.z) * g.gw + c.w;
      dst_row = static_cast<char*>(ep.out) + slot * ep.ldo * ce;
      if (blockIdx.x == 0 && tx == 0) {
        if (ep.observed) ep.observed[slot] = 1.0f;
        if (ep.age) ep.age[slot] = 0.0f;
      }
    }
    if (!dst_row) continue;
    for (int j = 0; j < 4; ++j) {
      const int col = n0 + tx * 4 + j;
      if (col >= g.D) continue;
      float v = valid ? acc[i][j] + (ep.bias ? ep.bias[col] : 0.0f) : 0.0f;
      if (valid && ep.position_table) {
        const int4 c = row_c[m];
        v = v + ep.position_table[(((int64_t)c.y * g.gh + c.z) * g.gw + c.w) * ep.pos_ld + col];
      }
      if (valid && ep.modality_embed) v = v + ep.modality_embed[col];
      if (ep.out_dtype == BJF_DTYPE_F32)
        reinterpret_cast<float*>(dst_row)[col] = v;
      else if (ep.out_dtype == BJF_DTYPE_F16)
        reinterpret_cast<__half*>(dst_row)[col] = __float2half_rn(v);
      else
        reinterpret_cast<__nv_bfloat16*>(dst_row)[col] = __float2bfloat16_rn(v);
    }
  }
}

// Output columns per tile: all of D up to 256, else D spread over the fewest tiles of at most
// 256 columns, rounded up to a multiple of 16 (the last column tile may be partial: its weight
// rows beyond D load as zeros and its columns beyond D are not stored).  Fewer, wider tiles
// gather A fewer times, which pays more than the MMA work on padding (D = 1408: six 256-column
// tiles ran the ViT-g batch 1.2x faster than eight of 176), and evening the tiles out trims that
// padding (six tiles of 240 rather than five of 256 and a half-padded sixth: 1.2 % faster).
int choose_bn(int D) {
  const int tiles = (D + kMaxBN - 1) / kMaxBN;
  return ((D + tiles - 1) / tiles + 15) / 16 * 16;
}

std::mutex g_attr_mu;
bool g_attr_set[64][2] = {};
// resident CTA-pair clusters per device, operand type and epilogue; the pair layouts take more
// than half an SM's shared memory, so one CTA per SM whatever the launch's stream count
int g_pair_clusters[64][4] = {};

}  // namespace

bool sm100_path_supported(const DeviceInfo& dev, const GatherGeometry& g, int32_t in_dt, int32_t w_dt,
                          const void* input, const void* weight) {
  if (dev.cc_major != 10) return false;
  if (in_dt != w_dt || (in_dt != BJF_DTYPE_F16 && in_dt != BJF_DTYPE_BF16)) return false;
  if (g.pw % 8 != 0 || g.W % 8 != 0) return false;
  if (g.K % kBK != 0 || g.K / kBK > kMaxKBlocks) return false;
  if (reinterpret_cast<uintptr_t>(input) % 16 != 0 || reinterpret_cast<uintptr_t>(weight) % 16 != 0)
    return false;
  if (dev.max_smem_optin < (size_t)SmemLayout::alloc ||
      dev.max_smem_optin < PairSmemLayout<true>::bytes(kMaxKBlocks, kMaxRowStreams))
    return false;
  return true;
}

// ---- split K for small row counts ----------------------------------------------------------
//
// A plain GEMM with fewer 256 x bn tiles than half the CTA pairs leaves most SMs idle while each
// tile walks the whole K loop.  Then each tile becomes ks units over K ranges of num_kb / ks
// blocks (ks a divisor of num_kb, at least four blocks a unit); every unit writes its f32 partial
// sums to its own slice of a scratch buffer, and splitk_reduce_kernel adds the slices in a fixed
// order, then the bias, and writes the output (zeros for rows outside the grid, as the epilogue
// does), so results do not depend on timing.
int choose_ksplit(int64_t pair_tiles, int max_clusters, int num_kb) {
  if (pair_tiles <= 0 || pair_tiles * 2 > max_clusters) return 1;
  const int64_t want = max_clusters / pair_tiles;
  int best = 1;
  for (int k = 2; k <= want && k <= num_kb; ++k)
    if (num_kb % k == 0 && num_kb / k >= 4) best = k;
  return best;
}

// out[m, 4q .. 4q + 3] from the ks partial slices; one thread per four columns (D % 4 == 0).
template <typename O>
__global__ void __launch_bounds__(256)
    splitk_reduce_kernel(const float* __restrict__ part, int ks, int64_t slice, const RowSource rs,
                         const int32_t* __restrict__ rows_dev, int rows_cap, GatherGeometry g, EpilogueArgs ep) {
  pdl_wait();
  int M = rows_cap;
  if (rows_dev) M = min(M, max(0, __ldg(rows_dev)));
  const int d4 = g.D / 4;
  const int64_t total = (int64_t)M * d4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int m = (int)(i / d4), d = (int)(i - (int64_t)m * d4) * 4;
    bool valid = false;
    row_base_offset(g, __ldg(rs.coords + m), valid);
    float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (valid) {
      v = __ldg(reinterpret_cast<const float4*>(part + (int64_t)m * g.D + d));
      for (int k = 1; k < ks; ++k) {
        const float4 p = __ldg(reinterpret_cast<const float4*>(part + k * slice + (int64_t)m * g.D + d));
        v.x = v.x + p.x;
        v.y = v.y + p.y;
        v.z = v.z + p.z;
        v.w = v.w + p.w;
      }
      if (ep.bias) {
        const float4 b = __ldg(reinterpret_cast<const float4*>(ep.bias + d));
        v.x = v.x + b.x;
        v.y = v.y + b.y;
        v.z = v.z + b.z;
        v.w = v.w + b.w;
      }
    }
    O* o = reinterpret_cast<O*>(static_cast<char*>(ep.out) + ((int64_t)m * ep.ldo + d) * (int64_t)sizeof(O));
    o[0] = from_f32<O>(v.x);
    o[1] = from_f32<O>(v.y);
    o[2] = from_f32<O>(v.z);
    o[3] = from_f32<O>(v.w);
  }
}

// ---- f32 operands on the tensor cores: an error-compensated bf16 split ----------------------
//
// x = hi + lo with hi = bf16(x) and lo = bf16(x - hi) (x - hi is exact in f32), so hi + lo
// carries 16 significant bits and |x - hi - lo| <= 2^-17 |x|.  Per product
// a w = a_hi w_hi + a_hi w_lo + a_lo w_hi + O(2^-16 |a w|): three bf16 products, each exact in
// the f32 accumulator.  The three run as one bf16 GEMM over K' = 3K by tripling the channel
// axis: the gathered rows as [a_hi | a_hi | a_lo] and the weight as [w_hi | w_lo | w_hi], channel
// groups in K order (the channel is K's slowest axis).  split_rows_part writes the split rows
// into a bf16 copy of the input with 3C channels at the same (b, t, r, col) positions, so the
// GEMM reads it with the caller's own rows and epilogue (plain, encoder input or cache scatter).
// Only the selected tubelets of that copy are written, and only they are read.

__device__ __forceinline__ uint32_t bf162_bits(__nv_bfloat162 v) {
  return (uint32_t)__bfloat16_as_ushort(v.x) | ((uint32_t)__bfloat16_as_ushort(v.y) << 16);
}
__device__ __forceinline__ void split_bf16x2(float a, float b, uint32_t& hi, uint32_t& lo) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);  // .x = a's, the low half
  const float2 hf = __bfloat1622float2(h);
  hi = bf162_bits(h);
  lo = bf162_bits(__floats2bfloat162_rn(a - hf.x, b - hf.y));
}
__device__ __forceinline__ void split_bf16x4(float4 x, uint2& hi, uint2& lo) {
  split_bf16x2(x.x, x.y, hi.x, lo.x);
  split_bf16x2(x.z, x.w, hi.y, lo.y);
}

// weight [D, K] f32 -> [D, 3K] bf16 as [hi | lo | hi] per row; K % 4 == 0.
// The weight split by blocks [0, nblocks) of a launch (this is block `bid`).
__device__ __forceinline__ void split_weight_part(const float* __restrict__ w, int D, int K,
                                                  __nv_bfloat16* __restrict__ w3, int bid, int nblocks) {
  const int64_t n4 = (int64_t)D * (K / 4);
  for (int64_t i = bid * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)nblocks * blockDim.x) {
    const int64_t d = i / (K / 4), k = (i - d * (K / 4)) * 4;
    uint2 hi, lo;
    split_bf16x4(__ldg(reinterpret_cast<const float4*>(w + d * K + k)), hi, lo);
    uint2* row = reinterpret_cast<uint2*>(w3 + d * 3 * K + k);
    row[0] = hi;
    row[K / 4] = lo;
    row[K / 2] = hi;
  }
}

// The rows of `rs` (as the GEMM resolves them) from the f32 input into a bf16 input of 3C
// channels, one warp per row, four consecutive k (inside one pw run, pw % 4 == 0) per lane.
// Rows outside the grid are skipped, as the GEMM reads them as zeros.
// By blocks [0, nblocks) of a launch (this is block `bid`); block-wide (`soff`: kMaxRowStreams + 1
// ints of shared memory).
__device__ __forceinline__ void split_rows_part(const float* __restrict__ video, const RowSource& rs,
                                                const int32_t* __restrict__ rows_dev, int rows_cap,
                                                const GatherGeometry& g, __nv_bfloat16* __restrict__ pv, int* soff,
                                                int bid, int nblocks) {
  pdl_wait();  // the rows come from the kernels before, and `pv` may be memory they read
  int M = rows_cap;
  if (rows_dev) M = min(M, max(0, __ldg(rows_dev)));
  M = min(M, load_row_offsets(rs, soff));
  const int lane = threadIdx.x & 31, wpb = blockDim.x >> 5;
  const int64_t plane = (int64_t)g.Ts * g.H * g.W;  // one channel of one batch element
  for (int m = bid * wpb + (threadIdx.x >> 5); m < M; m += nblocks * wpb) {
    bool valid = false;
    const int4 c = fetch_row(rs, soff, g, m);
    const int64_t base = row_base_offset(g, c, valid);
    if (!valid) continue;
    const int64_t pbase = base + (int64_t)c.x * 2 * g.C * plane;  // batch stride 3C planes
    // four loads in flight per lane before their splits and stores
    for (int k0 = lane * 4; k0 < g.K; k0 += 4 * 128) {
      float4 x[4];
      int64_t ko[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int k = k0 + u * 128;
        ko[u] = k < g.K ? k_offset(g, k) : -1;
        if (ko[u] >= 0) x[u] = __ldg(reinterpret_cast<const float4*>(video + base + ko[u]));
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (ko[u] < 0) continue;
        uint2 hi, lo;
        split_bf16x4(x[u], hi, lo);
        *reinterpret_cast<uint2*>(pv + pbase + ko[u]) = hi;
        *reinterpret_cast<uint2*>(pv + pbase + ko[u] + g.C * plane) = hi;
        *reinterpret_cast<uint2*>(pv + pbase + ko[u] + 2 * g.C * plane) = lo;
      }
    }
  }
}

// Both splits in one launch: blocks [0, wblocks) split the weight, the rest the rows, so the two
// memory-bound passes share the device instead of running one after the other.  Every block
// waits for the kernels before it (as a programmatic dependent): the row blocks read their rows,
// and the split buffers come from the stream-ordered pool, whose memory an earlier GEMM of the
// stream may have been reading.
__global__ void __launch_bounds__(256) split_operands_kernel(const float* __restrict__ weight, int wblocks,
                                                             __nv_bfloat16* __restrict__ w3,
                                                             const float* __restrict__ video, const RowSource rs,
                                                             const int32_t* __restrict__ rows_dev, int rows_cap,
                                                             GatherGeometry g, __nv_bfloat16* __restrict__ pv) {
  __shared__ int soff[kMaxRowStreams + 1];
  if ((int)blockIdx.x < wblocks) {
    pdl_wait();
    split_weight_part(weight, g.D, g.K, w3, (int)blockIdx.x, wblocks);
    return;
  }
  split_rows_part(video, rs, rows_dev, rows_cap, g, pv, soff, (int)blockIdx.x - wblocks, (int)gridDim.x - wblocks);
}

// Whether f32 operands take the split: the bf16 path must take the tripled geometry, and the
// vector accesses need 16-byte aligned inputs with pw and W multiples of 8.
bool split_f32_supported(const DeviceInfo& dev, const GatherGeometry& g, const void* input, const void* weight) {
  if (dev.cc_major != 10 || g.pw % 8 != 0 || g.W % 8 != 0) return false;
  if (reinterpret_cast<uintptr_t>(input) % 16 != 0 || reinterpret_cast<uintptr_t>(weight) % 16 != 0) return false;
  const int64_t K3 = 3 * (int64_t)g.K;
  if (K3 % kBK != 0 || K3 / kBK > kMaxKBlocks) return false;
  const int64_t Ts = g.ring ? g.Ts : g.T;
  if (3 * (int64_t)g.C * Ts * g.H * g.W >= (int64_t(1) << 31)) return false;
  return dev.max_smem_optin >= (size_t)SmemLayout::alloc &&
         dev.max_smem_optin >= PairSmemLayout<true>::bytes(kMaxKBlocks, kMaxRowStreams);
}

bjf_status launch_split_f32(const DeviceInfo& dev, const float* input, const float* weight, const GatherGeometry& g0,
                            const RowSource& rows, const int32_t* rows_dev, int64_t rows_cap,
                            const EpilogueArgs& ep, cudaStream_t st, bool pdl) {
  GatherGeometry g = g0;
  if (!g.ring) g.Ts = g.T;
  const int64_t plane = (int64_t)g.Ts * g.H * g.W;
  const size_t pv_bytes = (size_t)g.batch * 3 * g.C * plane * sizeof(__nv_bfloat16);
  const size_t w_bytes = (size_t)g.D * 3 * g.K * sizeof(__nv_bfloat16);
  void* pv = nullptr;
  void* w3 = nullptr;
  bjf_status rc = stream_alloc(dev.device, pv_bytes, st, &pv);
  if (rc) return rc;
  rc = stream_alloc(dev.device, w_bytes, st, &w3);
  if (rc) {
    stream_free(pv, st);
    return rc;
  }
  const int sms = dev.sm_count > 0 ? dev.sm_count : 148;
  const int64_t w4 = (int64_t)g.D * (g.K / 4);
  const int wblocks = (int)std::min<int64_t>(ceil_div(w4, 256), sms);  // one block an SM for the weight
  const int rblocks = (int)std::min<int64_t>(ceil_div(rows_cap, 8), 8 * sms);
  {
    const cudaError_t e = launch_kernel(pdl, split_operands_kernel, dim3((unsigned)(wblocks + rblocks)), dim3(256),
                                        0, st, weight, wblocks, static_cast<__nv_bfloat16*>(w3), input, rows,
                                        rows_dev, (int)rows_cap, g, static_cast<__nv_bfloat16*>(pv));
    rc = e == cudaSuccess ? BJF_OK : cuda_status(e, "f32 operand split launch");
  }
  if (!rc) {
    GatherGeometry g3 = g;
    g3.C = 3 * g.C;
    g3.K = 3 * g.K;
    rc = launch_gather_gemm(dev, pv, BJF_DTYPE_BF16, w3, BJF_DTYPE_BF16, g3, rows, rows_dev, rows_cap, ep, st,
                            /*pdl=*/true);
  }
  // stream-ordered: the memory returns to the pool once the GEMM has finished with it
  const bjf_status f1 = stream_free(w3, st), f2 = stream_free(pv, st);
  return rc ? rc : (f1 ? f1 : f2);
}

bjf_status launch_gather_gemm(const DeviceInfo& dev, const void* input, int32_t in_dt,
                              const void* weight, int32_t w_dt, const GatherGeometry& g0,
                              const RowSource& rows, const int32_t* rows_dev, int64_t rows_cap,
                              const EpilogueArgs& ep, cudaStream_t st, bool pdl, bool may_allocate) {
  if (!rows.coords && (rows.streams <= 0 || rows.streams > kMaxRowStreams || !rows.indices || !rows.counts))
    return fail(BJF_ERR_INVALID_ARGUMENT, "gather-GEMM index rows need 1..4096 streams, indices and counts");
  if (rows_cap <= 0 || g0.D <= 0) return BJF_OK;
  if (in_dt == BJF_DTYPE_F32 && w_dt == BJF_DTYPE_F32 && may_allocate && split_f32_supported(dev, g0, input, weight))
    return launch_split_f32(dev, static_cast<const float*>(input), static_cast<const float*>(weight), g0, rows,
                            rows_dev, rows_cap, ep, st, pdl);
  GatherGeometry g = g0;
  g.num_kb = g.K / kBK;
  g.is_bf16 = in_dt == BJF_DTYPE_BF16;
  const BoundedWait bw = bounded_wait();
  g.wait_ns = bw.limit_ns;
  g.stall = bw.stall;
  if (!g.ring) g.Ts = g.T;
  if (sm100_path_supported(dev, g, in_dt, w_dt, input, weight) &&
      (int64_t)g.C * g.Ts * g.H * g.W < (int64_t(1) << 31)) {
    EncodeTiledFn encode = nullptr;
    bjf_status rc = encode_tiled_fn(&encode);
    if (rc) return rc;
    const int bn = choose_bn(g.D);
    CUtensorMap map;
    cuuint64_t dims[2] = {(cuuint64_t)g.K, (cuuint64_t)g.D};
    cuuint64_t strides[1] = {(cuuint64_t)g.K * 2};
    cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)bn};
    cuuint32_t estr[2] = {1, 1};
    CUresult cr = encode(&map, g.is_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                         2, const_cast<void*>(weight), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS)
      return fail(BJF_ERR_CUDA, "cuTensorMapEncodeTiled(weight) failed with code " + std::to_string((int)cr));
    const int slot = g.is_bf16 ? 1 : 0;
    // CTA pairs whenever there is more than one 128-row tile of rows
    const bool pair = rows_cap > kBM && (bn / 2) % 8 == 0;
    if (pair) {
      cuuint32_t pbox[2] = {(cuuint32_t)kBK, (cuuint32_t)(bn / 2)};
      cr = encode(&map, g.is_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  const_cast<void*>(weight), dims, strides, pbox, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (cr != CUDA_SUCCESS)
        return fail(BJF_ERR_CUDA, "cuTensorMapEncodeTiled(weight) failed with code " + std::to_string((int)cr));
      const bool embed = ep.position_table || ep.modality_embed;
      const int pslot = slot + (embed ? 2 : 0);
      const int streams = rows.coords ? 0 : rows.streams;
      const size_t smem_bytes = embed ? PairSmemLayout<true>::bytes(g.num_kb, streams)
                                      : PairSmemLayout<false>::bytes(g.num_kb, streams);
      const void* fn =
          g.is_bf16 ? (embed ? (const void*)gather_gemm_sm100_pair_kernel<__nv_bfloat16, true>
                             : (const void*)gather_gemm_sm100_pair_kernel<__nv_bfloat16, false>)
                    : (embed ? (const void*)gather_gemm_sm100_pair_kernel<__half, true>
                             : (const void*)gather_gemm_sm100_pair_kernel<__half, false>);
      int max_clusters = 0;
      {
        std::lock_guard<std::mutex> lock(g_attr_mu);
        if (!g_pair_clusters[dev.device][pslot]) {
          cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)PairSmemLayout<true>::bytes(kMaxKBlocks, kMaxRowStreams));
          if (e != cudaSuccess) return cuda_status(e, "gather-GEMM pair smem attribute");
          cudaLaunchConfig_t cfg = {};
          cudaLaunchAttribute attr[1];
          attr[0].id = cudaLaunchAttributeClusterDimension;
          attr[0].val.clusterDim.x = 2;
          attr[0].val.clusterDim.y = 1;
          attr[0].val.clusterDim.z = 1;
          cfg.gridDim = dim3(2 * (unsigned)std::max(1, dev.sm_count / 2));
          cfg.blockDim = dim3(kThreads);
          cfg.dynamicSmemBytes = smem_bytes;
          cfg.attrs = attr;
          cfg.numAttrs = 1;
          e = cudaOccupancyMaxActiveClusters(&max_clusters, fn, &cfg);
          if (e != cudaSuccess) return cuda_status(e, "gather-GEMM pair occupancy");
          if (max_clusters <= 0) return fail(BJF_ERR_CUDA, "gather-GEMM pair kernel cannot be resident");
          g_pair_clusters[dev.device][pslot] = max_clusters;
        }
        max_clusters = g_pair_clusters[dev.device][pslot];
      }
      const int64_t pair_tiles_cap = ceil_div(g.D, bn) * ceil_div(rows_cap, 2 * kBM);
      EpilogueArgs epk = ep;
      void* scratch = nullptr;
      int ks = 1;
      if (rows.coords && ep.mode == kEpiloguePlain && !embed && may_allocate && g.D % 4 == 0 &&
          (reinterpret_cast<uintptr_t>(ep.bias) & 15) == 0)
        ks = choose_ksplit(pair_tiles_cap, max_clusters, g.num_kb);
      const int64_t slice = rows_cap * (int64_t)g.D;  // f32 elements of one split's partials
      if (ks > 1) {
        bjf_status arc = stream_alloc(dev.device, (size_t)ks * slice * sizeof(float), st, &scratch);
        if (arc) return arc;
        g.ksplit = ks;
        epk.out = scratch;
        epk.out_dtype = BJF_DTYPE_F32;
        epk.out_elem_bytes = 4;
        epk.ldo = g.D;
        epk.bias = nullptr;
        epk.split_stride = slice * (int64_t)sizeof(float);
      } else {
        g.ksplit = 1;
      }
      const unsigned clusters = (unsigned)std::min<int64_t>(pair_tiles_cap * ks, max_clusters);
      cudaLaunchConfig_t cfg = {};
      cudaLaunchAttribute attr[2];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[1].val.programmaticStreamSerializationAllowed = 1;
      cfg.gridDim = dim3(2 * clusters);
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = smem_bytes;
      cfg.stream = st;
      cfg.attrs = attr;
      cfg.numAttrs = pdl ? 2 : 1;
      auto launch_pair = [&](auto kern, auto* typed_input) {
        return cudaLaunchKernelEx(&cfg, kern, map, typed_input, rows, rows_dev, (int)rows_cap, g, bn, epk,
                                  dev.error_flag);
      };
      cudaError_t e;
      if (g.is_bf16) {
        const auto* in = static_cast<const __nv_bfloat16*>(input);
        e = embed ? launch_pair(gather_gemm_sm100_pair_kernel<__nv_bfloat16, true>, in)
                  : launch_pair(gather_gemm_sm100_pair_kernel<__nv_bfloat16, false>, in);
      } else {
        const auto* in = static_cast<const __half*>(input);
        e = embed ? launch_pair(gather_gemm_sm100_pair_kernel<__half, true>, in)
                  : launch_pair(gather_gemm_sm100_pair_kernel<__half, false>, in);
      }
      bjf_status rc2 = e == cudaSuccess ? BJF_OK : cuda_status(e, "gather-GEMM (tcgen05 pair) launch");
      if (ks > 1) {
        if (!rc2) {
          const int64_t work = rows_cap * (g.D / 4);
          const unsigned rgrid = (unsigned)std::min<int64_t>(ceil_div(work, 256), 8LL * std::max(1, dev.sm_count));
          const float* part = static_cast<const float*>(scratch);
          if (ep.out_dtype == BJF_DTYPE_F32)
            e = launch_kernel(true, splitk_reduce_kernel<float>, dim3(rgrid), dim3(256), 0, st, part, ks, slice,
                              rows, rows_dev, (int)rows_cap, g, ep);
          else if (ep.out_dtype == BJF_DTYPE_F16)
            e = launch_kernel(true, splitk_reduce_kernel<__half>, dim3(rgrid), dim3(256), 0, st, part, ks, slice,
                              rows, rows_dev, (int)rows_cap, g, ep);
          else
            e = launch_kernel(true, splitk_reduce_kernel<__nv_bfloat16>, dim3(rgrid), dim3(256), 0, st, part, ks,
                              slice, rows, rows_dev, (int)rows_cap, g, ep);
          rc2 = e == cudaSuccess ? BJF_OK : cuda_status(e, "split-K reduce launch");
        }
        const bjf_status frc = stream_free(scratch, st);  // after the reduce, in stream order
        if (!rc2) rc2 = frc;
      }
      return rc2;
    }
    {
      std::lock_guard<std::mutex> lock(g_attr_mu);
      if (!g_attr_set[dev.device][slot]) {
        const void* fn = g.is_bf16 ? (const void*)gather_gemm_sm100_kernel<__nv_bfloat16>
                                   : (const void*)gather_gemm_sm100_kernel<__half>;
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, SmemLayout::alloc);
        if (e != cudaSuccess) return cuda_status(e, "gather-GEMM smem attribute");
        g_attr_set[dev.device][slot] = true;
      }
    }
    const int64_t tiles_cap = ceil_div(g.D, bn) * ceil_div(rows_cap, kBM);
    dim3 grid((unsigned)std::min<int64_t>(tiles_cap, dev.sm_count > 0 ? dev.sm_count : 148));
    cudaError_t e;
    if (g.is_bf16)
      e = launch_kernel(pdl, gather_gemm_sm100_kernel<__nv_bfloat16>, grid, dim3(kThreads), SmemLayout::alloc, st,
                        map, static_cast<const __nv_bfloat16*>(input), rows, rows_dev, (int)rows_cap, g, bn, ep,
                        dev.error_flag);
    else
      e = launch_kernel(pdl, gather_gemm_sm100_kernel<__half>, grid, dim3(kThreads), SmemLayout::alloc, st, map,
                        static_cast<const __half*>(input), rows, rows_dev, (int)rows_cap, g, bn, ep,
                        dev.error_flag);
    return e == cudaSuccess ? BJF_OK : cuda_status(e, "gather-GEMM (tcgen05) launch");
  }
  dim3 grid((unsigned)ceil_div(g.D, kSBN), (unsigned)ceil_div(rows_cap, kSBM));
  bool ok = dispatch_float(in_dt, [&](auto itag) {
    dispatch_float(w_dt, [&](auto wtag) {
      cudaError_t e = launch_kernel(pdl, gather_gemm_simt_kernel<decltype(itag), decltype(wtag)>, grid,
                                    dim3(kSThreads), 0, st, static_cast<const decltype(itag)*>(input), rows,
                                    rows_dev, (int)rows_cap, g, static_cast<const decltype(wtag)*>(weight), ep);
      if (e != cudaSuccess) cuda_status(e, "gather-GEMM (SIMT) launch");
    });
  });
  if (!ok) return fail(BJF_ERR_INVALID_ARGUMENT, "input dtype must be f32, f16 or bf16");
  return check_launch("gather-GEMM (SIMT) launch");
}

}  // namespace bjf

using namespace bjf;

namespace {

bjf_status patchify_forward(const bjf_patchify_config* cfg, const void* input, bjf_dtype input_dtype,
                            const int64_t id[5], const int32_t* coords, int64_t rows, const void* weight,
                            bjf_dtype weight_dtype, const int64_t wd[5], const float* bias,
                            const float* position_table, const float* modality_embed, void* out,
                            bjf_dtype out_dtype, bjf_stream_t stream) {
  if (!cfg || !id || !wd) return fail(BJF_ERR_INVALID_ARGUMENT, "config and dims must not be null");
  const int64_t vals[8] = {cfg->in_channels, cfg->out_channels, cfg->frames, cfg->height,
                           cfg->width, cfg->tubelet_size, cfg->patch_h, cfg->patch_w};
  for (int64_t v : vals)
    if (v <= 0 || v > (1 << 30)) return fail(BJF_ERR_INVALID_ARGUMENT, "sparse patchify config fields must be positive");
  if (id[0] <= 0) return fail(BJF_ERR_INVALID_ARGUMENT, "sparse patchify batch must be nonzero");
  if (id[1] != cfg->in_channels || id[2] != cfg->frames || id[3] != cfg->height || id[4] != cfg->width)
    return fail(BJF_ERR_INVALID_ARGUMENT, "sparse patchify input dims " + dims_str(id, 5) +
                                              " do not match the config");
  if (wd[0] != cfg->out_channels || wd[1] != cfg->in_channels || wd[2] != cfg->tubelet_size ||
      wd[3] != cfg->patch_h || wd[4] != cfg->patch_w)
    return fail(BJF_ERR_INVALID_ARGUMENT, "sparse patchify weight dims " + dims_str(wd, 5) +
                                              " do not match the config");
  if (cfg->frames % cfg->tubelet_size || cfg->height % cfg->patch_h || cfg->width % cfg->patch_w)
    return fail(BJF_ERR_INVALID_ARGUMENT,
                "sparse patchify input frames/height/width must be divisible by the tubelet and patch sizes");
  if (rows < 0) return fail(BJF_ERR_INVALID_ARGUMENT, "sparse patchify rows must be non-negative");
  if (rows > INT32_MAX) return fail(BJF_ERR_UNSUPPORTED, "sparse patchify supports up to 2^31-1 rows");
  const int64_t K = cfg->in_channels * cfg->tubelet_size * cfg->patch_h * cfg->patch_w;
  if (K > (1 << 24) || cfg->out_channels > (1 << 24)) return fail(BJF_ERR_UNSUPPORTED, "sparse patchify K or D too large");
  if (dtype_size(out_dtype) == 0 || out_dtype == BJF_DTYPE_I32)
    return fail(BJF_ERR_INVALID_ARGUMENT, "output dtype must be f32, f16 or bf16");
  if (rows == 0) return BJF_OK;
  if (!input || !coords || !weight || !out) return fail(BJF_ERR_INVALID_ARGUMENT, "buffers must not be null");
  if (reinterpret_cast<uintptr_t>(coords) % 16) return fail(BJF_ERR_INVALID_ARGUMENT, "coords must be 16-byte aligned");
  const DeviceInfo* dev = nullptr;
  bjf_status rc = current_device(&dev);
  if (rc) return rc;
  GatherGeometry g{};
  g.C = (int)cfg->in_channels;
  g.T = (int)cfg->frames;
  g.H = (int)cfg->height;
  g.W = (int)cfg->width;
  g.kt = (int)cfg->tubelet_size;
  g.ph = (int)cfg->patch_h;
  g.pw = (int)cfg->patch_w;
  g.batch = (int)std::min<int64_t>(id[0], INT32_MAX);
  g.depth = g.T / g.kt;
  g.gh = g.H / g.ph;
  g.gw = g.W / g.pw;
  g.K = (int)K;
  g.D = (int)cfg->out_channels;
  EpilogueArgs ep{};
  ep.mode = kEpiloguePlain;
  ep.out = out;
  ep.out_dtype = out_dtype;
  ep.out_elem_bytes = (int)dtype_size(out_dtype);
  ep.ldo = g.D;
  ep.bias = bias;
  ep.position_table = position_table;
  ep.pos_ld = g.D;
  ep.modality_embed = modality_embed;
  return launch_gather_gemm(*dev, input, input_dtype, weight, weight_dtype, g,
                            coords_rows(reinterpret_cast<const int4*>(coords)), nullptr, rows, ep, as_cuda(stream));
}

}  // namespace

extern "C" bjf_status bjf_sparse_patchify3d_forward(const bjf_patchify_config* cfg, const void* input,
                                                    bjf_dtype input_dtype, const int64_t id[5],
                                                    const int32_t* coords, int64_t rows,
                                                    const void* weight, bjf_dtype weight_dtype,
                                                    const int64_t wd[5], const float* bias, void* out,
                                                    bjf_dtype out_dtype, bjf_stream_t stream) {
  return patchify_forward(cfg, input, input_dtype, id, coords, rows, weight, weight_dtype, wd, bias, nullptr, nullptr,
                          out, out_dtype, stream);
}

extern "C" bjf_status bjf_sparse_patchify3d_forward_encoder_input(
    const bjf_patchify_config* cfg, const void* input, bjf_dtype input_dtype, const int64_t id[5],
    const int32_t* coords, int64_t rows, const void* weight, bjf_dtype weight_dtype, const int64_t wd[5],
    const float* bias, const float* position_table, const float* modality_embed, void* out, bjf_dtype out_dtype,
    bjf_stream_t stream) {
  return patchify_forward(cfg, input, input_dtype, id, coords, rows, weight, weight_dtype, wd, bias, position_table,
                          modality_embed, out, out_dtype, stream);
}
