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
#include <string>

#include "common.cuh"
#include "status.hpp"

namespace bjf {
namespace {

constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads)
    age_observed_kernel(float* __restrict__ age, const float* __restrict__ observed, long long n) {
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
  long long i = (long long)blockIdx.x * kThreads + threadIdx.x;
  if (i < n) age[i] += observed[i];
}

// One warp per (b, s) row.  VECTOR: D % 8 == 0 and 16-byte aligned rows.
template <typename TokT, typename CacheT, bool VECTOR>
__global__ void __launch_bounds__(kThreads)
    scatter_rows_kernel(CacheT* __restrict__ features, float* __restrict__ observed,
                        float* __restrict__ age, const TokT* __restrict__ tokens,
                        const int32_t* __restrict__ token_indices, int sparse_len, int dense_tokens,
                        int embed_dim, long long rows) {
  long long row = (long long)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  const long long b = row / sparse_len;
  const int32_t idx = token_indices[row];
  if (idx < 0 || idx >= dense_tokens) return;
  const TokT* src = tokens + row * embed_dim;
  CacheT* dst = features + (b * dense_tokens + idx) * (long long)embed_dim;
  if (VECTOR) {
    for (int c = lane * 8; c < embed_dim; c += 32 * 8) {
      float v[8];
      load8<TokT>(src + c, v);
      store8<CacheT>(dst + c, v);
    }
  } else {
    for (int c = lane; c < embed_dim; c += 32) dst[c] = from_f32<CacheT>(to_f32<TokT>(src[c]));
  }
  if (lane == 0) {
    observed[b * dense_tokens + idx] = 1.0f;
    age[b * dense_tokens + idx] = 0.0f;
  }
}

template <typename TokT, typename CacheT>
void launch_scatter(bool vec, void* features, float* observed, float* age, const void* tokens,
                    const int32_t* idx, int S, int N, int D, long long rows, cudaStream_t st) {
  unsigned blocks = (unsigned)ceil_div(rows, kThreads / 32);
  if (vec)
    scatter_rows_kernel<TokT, CacheT, true><<<blocks, kThreads, 0, st>>>(
        static_cast<CacheT*>(features), observed, age, static_cast<const TokT*>(tokens), idx, S, N, D, rows);
  else
    scatter_rows_kernel<TokT, CacheT, false><<<blocks, kThreads, 0, st>>>(
        static_cast<CacheT*>(features), observed, age, static_cast<const TokT*>(tokens), idx, S, N, D, rows);
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
                                        bool age_observed, cudaStream_t st) {
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
  bool handled = dispatch_float(tdt, [&](auto ttag) {
    dispatch_float(fdt, [&](auto ctag) {
      launch_scatter<decltype(ttag), decltype(ctag)>(vec, features, observed, age, tokens, idx,
                                                      (int)S, (int)N, (int)D, rows, st);
    });
  });
  if (!handled) return fail(BJF_ERR_INVALID_ARGUMENT, "token dtype must be f32, f16 or bf16");
  return check_launch("feature memory scatter launch");
}

}  // namespace bjf

using namespace bjf;

extern "C" bjf_status bjf_feature_memory_assign_latest(
    void* features, bjf_dtype features_dtype, const int64_t fd[3], float* observed,
    const int64_t od[2], float* age_frames, const int64_t ad[2], const void* tokens,
    bjf_dtype tokens_dtype, const int64_t td[3], const int32_t* token_indices, const int64_t id[2],
    int32_t age_observed, bjf_stream_t stream) {
  if (!fd || !od || !ad || !td || !id) return fail(BJF_ERR_INVALID_ARGUMENT, "tensor dims must not be null");
  const int64_t batch = fd[0], dense = fd[1], dim = fd[2];
  // Messages and check order follow src/sparse_feature_memory.rs:124-178.
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
  return feature_memory_assign_launch(features, features_dtype, observed, age_frames, tokens,
                                      tokens_dtype, token_indices, batch, dense, dim, sparse_len,
                                      age_observed != 0, as_cuda(stream));
}
