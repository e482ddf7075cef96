// th_attention: flash attention (online softmax, never materialising the
// [S, S] score matrix) over token-major q/k/v, with causal masking and
// grouped-query heads.  This is the fp32-accumulating CUDA-core kernel: it
// serves fp32 models exactly and is the correctness baseline for the 2-byte
// types.  Semantics follow the reference `attention` op
// (src/torch_helion/optimizer/evaluate.py:139-146): softmax(q k^T * scale) v
// per (batch, head), here additionally masked to j <= i when causal.
#include <float.h>

#include <type_traits>

#include "common.cuh"

namespace th {

constexpr int AT_BQ = 64, AT_BK = 64;

template <typename T, int D>
__global__ void __launch_bounds__(256) attention_simt_kernel(th_attention_args p) {
  extern __shared__ float sm[];
  float* Qs = sm;                       // [BQ][D+1]
  float* Ks = Qs + AT_BQ * (D + 1);     // [BK][D+1]
  float* Vs = Ks + AT_BK * (D + 1);     // [BK][D]
  float* Ps = Vs + AT_BK * D;           // [BQ][BK+1]
  const int tid = threadIdx.x, r = tid >> 2, sub = tid & 3;
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int group = p.hq / p.hkv, hk = h / group;
  const int q0 = qb * AT_BQ;
  const T* q = reinterpret_cast<const T*>(p.q);
  const T* k = reinterpret_cast<const T*>(p.k);
  const T* v = reinterpret_cast<const T*>(p.v);
  T* o = reinterpret_cast<T*>(p.o);
  const int64_t tok0 = (int64_t)b * p.seq;
  for (int i = tid; i < AT_BQ * D; i += 256) {
    const int rr = i / D, dd = i % D, s = q0 + rr;
    Qs[rr * (D + 1) + dd] = s < p.seq ? to_f32(q[(tok0 + s) * p.ldq + (int64_t)h * D + dd]) : 0.f;
  }
  const float sl2 = p.scale * 1.4426950408889634f;  // scores in log2 units
  float m = -FLT_MAX, l = 0.f;
  float acc[D / 4];
#pragma unroll
  for (int j = 0; j < D / 4; ++j) acc[j] = 0.f;
  const int qi = q0 + r;
  int kv_end = p.seq;
  if (p.causal) kv_end = min(p.seq, q0 + AT_BQ);
  for (int k0 = 0; k0 < kv_end; k0 += AT_BK) {
    __syncthreads();
    for (int i = tid; i < AT_BK * D; i += 256) {
      const int rr = i / D, dd = i % D, s = k0 + rr;
      const bool ok = s < p.seq;
      Ks[rr * (D + 1) + dd] = ok ? to_f32(k[(tok0 + s) * p.ldk + (int64_t)hk * D + dd]) : 0.f;
      Vs[rr * D + dd] = ok ? to_f32(v[(tok0 + s) * p.ldv + (int64_t)hk * D + dd]) : 0.f;
    }
    __syncthreads();
    float s16[AT_BK / 4];
    float mx = -FLT_MAX;
#pragma unroll
    for (int jj = 0; jj < AT_BK / 4; ++jj) {
      const int c = sub + 4 * jj, kj = k0 + c;
      float s = 0.f;
#pragma unroll 8
      for (int dd = 0; dd < D; ++dd) s = fmaf(Qs[r * (D + 1) + dd], Ks[c * (D + 1) + dd], s);
      const bool masked = kj >= p.seq || (p.causal && kj > qi);
      s = masked ? -FLT_MAX : s * sl2;
      s16[jj] = s;
      mx = fmaxf(mx, s);
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m, mx);
    const float alpha = (m == -FLT_MAX) ? 0.f : exp2f(m - m_new);
    float ls = 0.f;
#pragma unroll
    for (int jj = 0; jj < AT_BK / 4; ++jj) {
      const float pv = s16[jj] == -FLT_MAX ? 0.f : exp2f(s16[jj] - m_new);
      ls += pv;
      Ps[r * (AT_BK + 1) + sub + 4 * jj] = pv;
    }
    ls += __shfl_xor_sync(0xffffffffu, ls, 1);
    ls += __shfl_xor_sync(0xffffffffu, ls, 2);
    l = l * alpha + ls;
    m = m_new;
    __syncwarp();
#pragma unroll
    for (int j = 0; j < D / 4; ++j) acc[j] *= alpha;
    for (int c = 0; c < AT_BK; ++c) {
      const float pc = Ps[r * (AT_BK + 1) + c];
#pragma unroll
      for (int j = 0; j < D / 4; ++j) acc[j] = fmaf(pc, Vs[c * D + sub + 4 * j], acc[j]);
    }
  }
  if (qi < p.seq) {
    const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
    for (int j = 0; j < D / 4; ++j) o[(tok0 + qi) * p.ldo + (int64_t)h * D + sub + 4 * j] = from_f32<T>(acc[j] * inv);
  }
}

template <typename T, int D>
static int launch_attention(const th_attention_args* a, cudaStream_t st) {
  const size_t smem = sizeof(float) * (AT_BQ * (D + 1) + AT_BK * (D + 1) + AT_BK * D + AT_BQ * (AT_BK + 1));
  if (int rc = smem_limit(attention_simt_kernel<T, D>, smem, "th_attention")) return rc;
  dim3 grid((unsigned)((a->seq + AT_BQ - 1) / AT_BQ), (unsigned)a->hq, (unsigned)a->batch);
  attention_simt_kernel<T, D><<<grid, 256, smem, st>>>(*a);
  return check_launch("th_attention");
}

}  // namespace th

#include "attention_tc.cu"  // tcgen05 path for bf16/fp16, head_dim 64/128

namespace th {

template <typename T>
static int attention_dispatch(const th_attention_args* a, cudaStream_t st) {
  if constexpr (!std::is_same<T, float>::value) {
    int rc = TH_OK;
    if (attention_tc_try<T>(a, st, &rc) == 0) return rc;
  }
  switch (a->head_dim) {
    case 16: return launch_attention<T, 16>(a, st);
    case 32: return launch_attention<T, 32>(a, st);
    case 64: return launch_attention<T, 64>(a, st);
    case 128: return launch_attention<T, 128>(a, st);
    default: return fail(TH_EUNSUPPORTED, "th_attention: head_dim %d not built (16/32/64/128)", a->head_dim);
  }
}

}  // namespace th

extern "C" int th_attention(const th_attention_args* a, void* stream) {
  using namespace th;
  if (!a || !a->q || !a->k || !a->v || !a->o) return fail(TH_EINVAL, "th_attention: NULL argument");
  if (a->batch <= 0 || a->seq <= 0 || a->hq <= 0 || a->hkv <= 0 || a->hq % a->hkv)
    return fail(TH_EINVAL, "th_attention: bad heads/shape (hq %% hkv must be 0)");
  const int64_t d = a->head_dim;
  if (a->ldq < a->hq * d || a->ldo < a->hq * d || a->ldk < a->hkv * d || a->ldv < a->hkv * d)
    return fail(TH_EINVAL, "th_attention: leading dimension too small");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (a->dtype) {
    case TH_F32: return attention_dispatch<float>(a, st);
    case TH_BF16: return attention_dispatch<__nv_bfloat16>(a, st);
    case TH_F16: return attention_dispatch<__half>(a, st);
    default: return fail(TH_EDTYPE, "th_attention: bad dtype %d", a->dtype);
  }
}
