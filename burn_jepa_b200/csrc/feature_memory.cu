// feature_memory.cu -- step 3 of the sparse front end: in-place AssignLatest
// write of new token rows into the persistent [B, N, D] token cache.
//
// The reference (burn_jepa src/sparse_feature_memory.rs:22-267) allocates a new
// cache every frame, copies the whole [B, N, D] cache into it
// (copy_feature_memory_kernel, traffic proportional to B*N*D whatever the
// sparsity) and then scatters the S new rows (sparse_assign_feature_memory_kernel).
// Here the cache is updated in place, so a frame costs only the S rows it writes
// plus the [B, N] metadata: an aging pass (age += observed when the memory has
// stepped before) and a row scatter in which one warp moves one token row with
// 16-byte vector accesses and sets observed = 1, age = 0 for the slot.
// Out-of-range indices are skipped exactly as the reference's guards do (:79-85).
//
// The EMA update mode (InterframeJepaFeatureUpdateMode::Ema, src/feature_memory.rs:240-258)
// and row resets (reset_rows, :348-375), which the reference runs on its portable tensor
// path, run here as the same in-place row kernels: an EMA row becomes
//   (prev (1 - alpha) + new alpha) observed + new (1 - observed)
// added to the cache as a delta, in the reference's f32 operation order (no contraction).
#include <algorithm>
#include <string>

#include "common.cuh"
#include "runtime.hpp"
#include "status.hpp"

namespace bjf {
namespace {

constexpr int kThreads = 256;

// The aging passes let the row scatter launched after them start at once (programmatic
// dependent launch): the scatter copies its rows meanwhile and waits for the aging only
// before it writes the rows' observed / age.
__global__ void __launch_bounds__(kThreads)
    age_observed_kernel(float* __restrict__ age, const float* __restrict__ observed, long long n) {
  pdl_trigger();
  long long i = (long long)blockIdx.x * kThreads + threadIdx.x;
  long long n4 = n >> 2;
  if (i < n4) {
    float4 a = reinterpret_cast<float4*>(age)[i];
    float4 o = reinterpret_cast<const float4*>(observed)[i];
    a.x += o.x; a.y += o.y; a.z += o.z; a.w += o.w;
    reinterpret_cast<float4*>(age)[i] = a;
  }
  long long tail = n4 * 4 + i;
  if (i < (n & 3)) age[tail] += observed[tail];
}

__global__ void __launch_bounds__(kThreads)
    age_observed_scalar_kernel(float* __restrict__ age, const float* __restrict__ observed, long long n) {
  pdl_trigger();
  long long i = (long long)blockIdx.x * kThreads + threadIdx.x;
  if (i < n) age[i] += observed[i];
}

// EMA blend of one element (src/feature_memory.rs:244-256): the reference computes
// previous (1 - alpha) + tokens alpha, mixes it with the first observation by the slot's
// observed value, and adds the difference to the cache.  Rounded as it does, step by step.
__device__ __forceinline__ float ema_element(float prev, float tok, float alpha, float one_minus_alpha, float obs,
                                             float first) {
  const float blended = __fadd_rn(__fmul_rn(prev, one_minus_alpha), __fmul_rn(tok, alpha));
  const float next = __fadd_rn(__fmul_rn(blended, obs), __fmul_rn(tok, first));
  return __fadd_rn(prev, __fsub_rn(next, prev));
}

// One warp per (b, s) row.  VECTOR: D % 8 == 0 and 16-byte aligned rows, each lane keeping up
// to four (EMA: two, of both rows) 16-byte segments in flight.  EMA: blend with the cached row
// instead of overwriting it.  The observed / age writes wait for the aging pass launched before
// this kernel (the wait returns at once when there is none).
template <typename TokT, typename CacheT, bool VECTOR, bool EMA>
__global__ void __launch_bounds__(kThreads)
    scatter_rows_kernel(CacheT* __restrict__ features, float* __restrict__ observed,
                        float* __restrict__ age, const TokT* __restrict__ tokens,
                        const int32_t* __restrict__ token_indices, int sparse_len, int dense_tokens,
                        int embed_dim, long long rows, float alpha) {
  const int lane = threadIdx.x & 31;
  // a grid of resident blocks whose warps stride over the rows: no tail wave
  for (long long row = (long long)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); row < rows;
       row += (long long)gridDim.x * (kThreads / 32)) {
  const long long b = row / sparse_len;
  const int32_t idx = token_indices[row];
  if (idx < 0 || idx >= dense_tokens) continue;
  const TokT* src = tokens + row * embed_dim;
  CacheT* dst = features + (b * dense_tokens + idx) * (long long)embed_dim;
  // the slot's observed value before this update (read by every lane before lane 0 sets it)
  const float obs = EMA ? observed[b * dense_tokens + idx] : 0.0f;
  const float first = __fadd_rn(-obs, 1.0f);
  const float oma = __fsub_rn(1.0f, alpha);
  __syncwarp();
  if (VECTOR) {
    constexpr int kSeg = EMA ? 2 : 4;  // 16-byte segments per lane in flight (EMA: of both rows)
    for (int c0 = lane * 8; c0 < embed_dim; c0 += 32 * 8 * kSeg) {
      float v[kSeg][8];
#pragma unroll
      for (int u = 0; u < kSeg; ++u)
        if (c0 + u * 256 < embed_dim) load8<TokT>(src + c0 + u * 256, v[u]);
      if (EMA) {
        float pv[kSeg][8];
#pragma unroll
        for (int u = 0; u < kSeg; ++u)
          if (c0 + u * 256 < embed_dim) load8<CacheT>(dst + c0 + u * 256, pv[u]);
#pragma unroll
        for (int u = 0; u < kSeg; ++u)
#pragma unroll
          for (int j = 0; j < 8; ++j) v[u][j] = ema_element(pv[u][j], v[u][j], alpha, oma, obs, first);
      }
#pragma unroll
      for (int u = 0; u < kSeg; ++u)
        if (c0 + u * 256 < embed_dim) store8<CacheT>(dst + c0 + u * 256, v[u]);
    }
  } else {
    for (int c = lane; c < embed_dim; c += 32) {
      float v = to_f32<TokT>(src[c]);
      if (EMA) v = ema_element(to_f32<CacheT>(dst[c]), v, alpha, oma, obs, first);
      dst[c] = from_f32<CacheT>(v);
    }
  }
  if (lane == 0) {
    pdl_wait();
    observed[b * dense_tokens + idx] = 1.0f;
    age[b * dense_tokens + idx] = 0.0f;
  }
  }
}

// Blocks of kThreads for `work_blocks` blocks of work: at most the resident 8 per SM.
unsigned resident_blocks(long long work_blocks) {
  const DeviceInfo* dev = nullptr;
  const int sms = current_device(&dev) == BJF_OK && dev->sm_count > 0 ? dev->sm_count : 148;
  return (unsigned)std::max<long long>(1, std::min<long long>(work_blocks, 8LL * sms));
}

// after_aging: the kernel before this one in the stream is this update's aging pass.
template <typename TokT, typename CacheT, bool EMA>
cudaError_t launch_scatter(bool vec, bool after_aging, void* features, float* observed, float* age,
                           const void* tokens, const int32_t* idx, int S, int N, int D, long long rows, float alpha,
                           cudaStream_t st) {
  const dim3 blocks(resident_blocks(ceil_div(rows, kThreads / 32)));
  if (vec)
    return launch_kernel(after_aging, scatter_rows_kernel<TokT, CacheT, true, EMA>, blocks, dim3(kThreads), 0, st,
                         static_cast<CacheT*>(features), observed, age, static_cast<const TokT*>(tokens), idx, S, N,
                         D, rows, alpha);
  return launch_kernel(after_aging, scatter_rows_kernel<TokT, CacheT, false, EMA>, blocks, dim3(kThreads), 0, st,
                       static_cast<CacheT*>(features), observed, age, static_cast<const TokT*>(tokens), idx, S, N, D,
                       rows, alpha);
}

// Zeroes the features, observed and age of the listed batch rows (out-of-range rows are
// skipped).  grid = (chunks, rows); 16-byte stores where the row allows.
__global__ void __launch_bounds__(kThreads)
    reset_rows_kernel(char* __restrict__ features, long long feature_row_bytes, float* __restrict__ observed,
                      float* __restrict__ age, int dense_tokens, const int32_t* __restrict__ rows, int batch) {
  const int r = rows[blockIdx.y];
  if (r < 0 || r >= batch) return;
  char* f = features + (long long)r * feature_row_bytes;
  const long long stride = (long long)gridDim.x * kThreads;
  const long long t0 = (long long)blockIdx.x * kThreads + threadIdx.x;
  if ((reinterpret_cast<uintptr_t>(f) & 15) == 0 && (feature_row_bytes & 15) == 0) {
    uint4* f4 = reinterpret_cast<uint4*>(f);
    for (long long i = t0; i < feature_row_bytes / 16; i += stride) f4[i] = make_uint4(0, 0, 0, 0);
  } else {
    for (long long i = t0; i < feature_row_bytes; i += stride) f[i] = 0;
  }
  float* o = observed + (long long)r * dense_tokens;
  float* a = age + (long long)r * dense_tokens;
  for (long long i = t0; i < dense_tokens; i += stride) {
    o[i] = 0.0f;
    a[i] = 0.0f;
  }
}

bool mul_ok(int64_t a, int64_t b, int64_t& out) {
  if (a < 0 || b < 0) return false;
  if (a != 0 && b > INT64_MAX / a) return false;
  out = a * b;
  return true;
}

}  // namespace

// Launches aging (when requested) then the row scatter; shapes already validated.
bjf_status feature_memory_assign_launch(void* features, int32_t fdt, float* observed, float* age,
                                        const void* tokens, int32_t tdt, const int32_t* idx,
                                        int64_t B, int64_t N, int64_t D, int64_t S,
                                        bool age_observed, cudaStream_t st, bool ema = false, float alpha = 0.0f) {
  const long long meta = (long long)(B * N);
  if (age_observed && meta > 0) {
    bool aligned = reinterpret_cast<uintptr_t>(age) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(observed) % 16 == 0;
    if (aligned) {
      long long work = (meta >> 2) > (meta & 3) ? (meta >> 2) : (meta & 3);
      age_observed_kernel<<<(unsigned)ceil_div(work, kThreads), kThreads, 0, st>>>(age, observed, meta);
    } else {
      age_observed_scalar_kernel<<<(unsigned)ceil_div(meta, kThreads), kThreads, 0, st>>>(age, observed, meta);
    }
    bjf_status rc = check_launch("feature memory aging launch");
    if (rc) return rc;
  }
  const long long rows = (long long)(B * S);
  if (rows == 0) return BJF_OK;
  const size_t fe = dtype_size(fdt), te = dtype_size(tdt);
  const bool vec = (D % 8 == 0) && reinterpret_cast<uintptr_t>(features) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(tokens) % 16 == 0 && (D * (int64_t)fe) % 16 == 0 &&
                   (D * (int64_t)te) % 16 == 0;
  const bool after_aging = age_observed && meta > 0;
  cudaError_t e = cudaSuccess;
  bool handled = dispatch_float(tdt, [&](auto ttag) {
    dispatch_float(fdt, [&](auto ctag) {
      if (ema)
        e = launch_scatter<decltype(ttag), decltype(ctag), true>(vec, after_aging, features, observed, age, tokens,
                                                                 idx, (int)S, (int)N, (int)D, rows, alpha, st);
      else
        e = launch_scatter<decltype(ttag), decltype(ctag), false>(vec, after_aging, features, observed, age, tokens,
                                                                  idx, (int)S, (int)N, (int)D, rows, alpha, st);
    });
  });
  if (!handled) return fail(BJF_ERR_INVALID_ARGUMENT, "token dtype must be f32, f16 or bf16");
  if (e != cudaSuccess) return cuda_status(e, "feature memory scatter launch");
  return check_launch("feature memory scatter launch");
}

}  // namespace bjf

using namespace bjf;

namespace {

// Shape validation of the sparse cache update; messages and check order follow
// src/sparse_feature_memory.rs:124-178.
bjf_status validate_update(void* features, bjf_dtype features_dtype, const int64_t fd[3], float* observed,
                           const int64_t od[2], float* age_frames, const int64_t ad[2], const void* tokens,
                           const int64_t td[3], const int32_t* token_indices, const int64_t id[2]) {
  if (!fd || !od || !ad || !td || !id) return fail(BJF_ERR_INVALID_ARGUMENT, "tensor dims must not be null");
  const int64_t batch = fd[0], dense = fd[1], dim = fd[2];
  if (od[0] != batch || od[1] != dense || ad[0] != batch || ad[1] != dense) {
    return fail(BJF_ERR_INVALID_ARGUMENT,
                "feature memory metadata dims mismatch: features=" + dims_str(fd, 3) +
                    " observed=" + dims_str(od, 2) + " age=" + dims_str(ad, 2));
  }
  if (td[0] != batch || td[2] != dim) {
    return fail(BJF_ERR_INVALID_ARGUMENT,
                "feature memory token dims mismatch: tokens=" + dims_str(td, 3) + " expected=[" +
                    std::to_string(batch) + ",sparse," + std::to_string(dim) + "]");
  }
  const int64_t sparse_len = td[1];
  if (id[0] != batch || id[1] != sparse_len) {
    return fail(BJF_ERR_INVALID_ARGUMENT,
                "feature memory index dims mismatch: indices=" + dims_str(id, 2) + " expected=[" +
                    std::to_string(batch) + "," + std::to_string(sparse_len) + "]");
  }
  if (sparse_len == 0)
    return fail(BJF_ERR_INVALID_ARGUMENT, "feature memory sparse assignment requires at least one token");
  int64_t fe, me, se, sm;
  if (!mul_ok(batch, dense, me) || !mul_ok(me, dim, fe))
    return fail(BJF_ERR_INVALID_ARGUMENT, "feature memory feature element count overflow");
  if (!mul_ok(batch, sparse_len, sm) || !mul_ok(sm, dim, se))
    return fail(BJF_ERR_INVALID_ARGUMENT, "feature memory sparse feature element count overflow");
  if (batch < 0 || dense < 0 || dim < 0 || sparse_len < 0)
    return fail(BJF_ERR_INVALID_ARGUMENT, "feature memory dims must be non-negative");
  if (dense > INT32_MAX || dim > INT32_MAX || sparse_len > INT32_MAX)
    return fail(BJF_ERR_UNSUPPORTED, "feature memory dims exceed the int32 index range");
  if (fe > 0 && (!features || !observed || !age_frames))
    return fail(BJF_ERR_INVALID_ARGUMENT, "feature memory buffers must not be null");
  if (se > 0 && (!tokens || !token_indices))
    return fail(BJF_ERR_INVALID_ARGUMENT, "token buffers must not be null");
  if (dtype_size(features_dtype) == 0 || features_dtype == BJF_DTYPE_I32)
    return fail(BJF_ERR_INVALID_ARGUMENT, "feature memory dtype must be f32, f16 or bf16");
  return BJF_OK;
}

}  // namespace

extern "C" bjf_status bjf_feature_memory_assign_latest(
    void* features, bjf_dtype features_dtype, const int64_t fd[3], float* observed,
    const int64_t od[2], float* age_frames, const int64_t ad[2], const void* tokens,
    bjf_dtype tokens_dtype, const int64_t td[3], const int32_t* token_indices, const int64_t id[2],
    int32_t age_observed, bjf_stream_t stream) {
  bjf_status rc = validate_update(features, features_dtype, fd, observed, od, age_frames, ad, tokens, td,
                                  token_indices, id);
  if (rc) return rc;
  return feature_memory_assign_launch(features, features_dtype, observed, age_frames, tokens, tokens_dtype,
                                      token_indices, fd[0], fd[1], fd[2], td[1], age_observed != 0, as_cuda(stream));
}

extern "C" bjf_status bjf_feature_memory_update_ema(
    void* features, bjf_dtype features_dtype, const int64_t fd[3], float* observed, const int64_t od[2],
    float* age_frames, const int64_t ad[2], const void* tokens, bjf_dtype tokens_dtype, const int64_t td[3],
    const int32_t* token_indices, const int64_t id[2], float alpha, int32_t age_observed, bjf_stream_t stream) {
  bjf_status rc = validate_update(features, features_dtype, fd, observed, od, age_frames, ad, tokens, td,
                                  token_indices, id);
  if (rc) return rc;
  // InterframeJepaFeatureMemoryConfig::normalized (src/feature_memory.rs:40-48): f32 clamp
  // to [0, 1] (a NaN stays NaN).
  if (alpha < 0.0f) alpha = 0.0f;
  if (alpha > 1.0f) alpha = 1.0f;
  return feature_memory_assign_launch(features, features_dtype, observed, age_frames, tokens, tokens_dtype,
                                      token_indices, fd[0], fd[1], fd[2], td[1], age_observed != 0, as_cuda(stream),
                                      true, alpha);
}

extern "C" bjf_status bjf_feature_memory_reset_rows(void* features, bjf_dtype features_dtype, const int64_t fd[3],
                                                    float* observed, float* age_frames, const int32_t* rows,
                                                    int64_t row_count, bjf_stream_t stream) {
  if (!fd) return fail(BJF_ERR_INVALID_ARGUMENT, "tensor dims must not be null");
  if (row_count < 0) return fail(BJF_ERR_INVALID_ARGUMENT, "row count must be non-negative");
  if (row_count == 0) return BJF_OK;  // reset_rows with no rows is a no-op (src/feature_memory.rs:349-352)
  if (row_count > 65535) return fail(BJF_ERR_UNSUPPORTED, "feature memory reset supports up to 65535 rows per call");
  const size_t fe = dtype_size(features_dtype);
  if (fe == 0 || features_dtype == BJF_DTYPE_I32)
    return fail(BJF_ERR_INVALID_ARGUMENT, "feature memory dtype must be f32, f16 or bf16");
  const int64_t batch = fd[0], dense = fd[1], dim = fd[2];
  int64_t nd = 0, row_bytes = 0;
  if (batch < 0 || dense < 0 || dim < 0 || !mul_ok(dense, dim, nd) || !mul_ok(nd, (int64_t)fe, row_bytes))
    return fail(BJF_ERR_INVALID_ARGUMENT, "feature memory dims must be non-negative");
  if (batch > INT32_MAX || dense > INT32_MAX) return fail(BJF_ERR_UNSUPPORTED, "feature memory dims exceed the int32 index range");
  if (!features || !observed || !age_frames || !rows)
    return fail(BJF_ERR_INVALID_ARGUMENT, "feature memory buffers must not be null");
  const long long work = std::max<long long>(row_bytes / 16, dense);
  const unsigned chunks = (unsigned)std::min<long long>(std::max<long long>(ceil_div(work, kThreads), 1), 1024);
  reset_rows_kernel<<<dim3(chunks, (unsigned)row_count), kThreads, 0, as_cuda(stream)>>>(
      static_cast<char*>(features), row_bytes, observed, age_frames, (int)dense, rows, (int)batch);
  return check_launch("feature memory reset launch");
}
