// tcgen05 flash attention (forward) for bf16/fp16, head_dim 64 or 128.
//
// One CTA = 128 query rows of one (batch, query head); KV blocks of 128 rows.
// 320 threads, warp-specialised:
//   warp 0    TMA: the Q tile once, then K and V tiles into separate 3-stage rings, in
//             the order the MMA warp consumes them (K_0, K_1, V_0, K_2, V_1, ...), so
//             the load of the next K block never waits for a P.V product
//   warp 1    MMA: S_j = Q K_j^T into one of two TMEM S buffers (so S_{j+1} is
//             computed while the softmax warps work on S_j), then O += P_j V_j with
//             P_j read from tensor memory (V is an MN-major shared-memory operand:
//             head_dim is its contiguous axis); S buffer j&1 is reused by S_{j+2}
//             once P_j V_j, which reads P_j out of it, has completed
//   warps 2-9 softmax, two threads per query row, each owning one half of the key
//             columns with its own running max, row sum and O accumulator
//             (O = O_0 + O_1, P_h V_h into O_h), so the halves never exchange
//             maxima inside the loop: read S_j from TMEM, masked online softmax
//             in the log2 domain, P_j (bf16 pairs) stored back into the first 32
//             columns of the thread's own 64-column part of the S_j buffer, where
//             the P.V MMA reads it as its A operand.  O_h is rescaled in TMEM
//             only when its running max grows by more than 2^8 (a lazy rescale:
//             P stays <= 256); the epilogue merges the halves once.
// Causal masking skips KV blocks above the diagonal and masks the diagonal
// block; grouped-query heads read K/V head h / (hq/hkv).  Rows of a tile that
// run past the sequence (into the next batch element) are masked.
// TMEM: S buffers at columns [0,128) and [128,256) (P_j of key half h in columns
// [h*64, h*64+32) of its buffer), O_0 at [256, 256+D), O_1 after it.
#include "common.cuh"

namespace th {

template <int D>
struct AtCfg {
  static constexpr int BM = 128, BN = 128;
  static constexpr int DA = D / 64;                // 64-column atoms of head_dim
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;      // one K or one V tile
  static constexpr int STAGES = 3;                 // K ring and V ring depth
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = Q_BYTES;
  static constexpr int OFF_V = OFF_K + STAGES * KV_BYTES;
  static constexpr int OFF_RED = OFF_V + STAGES * KV_BYTES;  // epilogue (max, sum) exchange of the halves
  static constexpr int OFF_BAR = OFF_RED + 2 * 128 * 4;
  static constexpr int SMEM = 1024 + OFF_BAR + 256;
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

template <typename T, int D>
__global__ void __launch_bounds__(320, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, th_attention_args p) {
  using C = AtCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_align<1024>(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);
  constexpr int NS = C::STAGES;
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;             // [NS]
  uint64_t* k_empty = k_full + NS;         // [NS]
  uint64_t* v_full = k_empty + NS;         // [NS]
  uint64_t* v_empty = v_full + NS;         // [NS]
  uint64_t* s_full = v_empty + NS;         // [2]
  uint64_t* s_free = s_full + 2;           // [2] S buffer (and the P in it) consumed by P.V
  uint64_t* p_full = s_free + 2;
  uint64_t* pv_done = p_full + 1;          // [2]
  uint64_t* mma_done = pv_done + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqb = (p.seq + C::BM - 1) / C::BM;
  const int qb = nqb - 1 - (int)blockIdx.x;  // heaviest (most KV blocks) first when causal
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.hq / p.hkv);
  const int q0 = qb * C::BM;
  const int64_t row0 = (int64_t)b * p.seq;
  const int nkv_all = (p.seq + C::BN - 1) / C::BN;
  const int nkv = p.causal ? min(nkv_all, (q0 + C::BM - 1) / C::BN + 1) : nkv_all;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_free[s], 1);
    }
    mbar_init(p_full, 8);
    mbar_init(&pv_done[0], 1);
    mbar_init(&pv_done[1], 1);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  __syncwarp();
  if (warp == 0) tmem_alloc(tslot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  pdl_wait();  // the previous kernel's outputs (this kernel's inputs) are complete
  pdl_trigger();
  const uint32_t tO = tmem + 256;

  if (warp == 0) {
    if (lane == 0) {  // ------------------------------------------- TMA
      mbar_arrive_expect_tx(q_full, C::Q_BYTES);
      for (int a = 0; a < C::DA; ++a)
        tma_load_2d(sm + C::OFF_Q + a * C::BM * 128, &tmQ, q_full, h * D + a * 64, (int)(row0 + q0));
      // one K or V tile of block j into its ring slot once the slot's previous reader is done
      auto load = [&](const CUtensorMap* tm, int off, uint64_t* full, uint64_t* empty, int j) -> bool {
        const int s = j % NS;
        if (!mbar_wait(&empty[s], ((j / NS) & 1) ^ 1, abort_flag)) return false;
        mbar_arrive_expect_tx(&full[s], C::KV_BYTES);
        for (int a = 0; a < C::DA; ++a)
          tma_load_2d(sm + off + s * C::KV_BYTES + a * C::BN * 128, tm, &full[s], hk * D + a * 64,
                      (int)(row0 + j * C::BN));
        return true;
      };
      // consumption order: S_0, S_1, PV_0, S_2, PV_1, ... -> loads K_0, K_1, V_0, K_2, V_1, K_3, V_2, ...
      bool ok = true;
      for (int j = 0; ok && j < min(nkv, 2); ++j) ok = load(&tmK, C::OFF_K, k_full, k_empty, j);
      if (ok && nkv > 0) ok = load(&tmV, C::OFF_V, v_full, v_empty, 0);
      for (int j = 0; ok && j + 1 < nkv; ++j) {
        if (j + 2 < nkv && !(ok = load(&tmK, C::OFF_K, k_full, k_empty, j + 2))) break;
        ok = load(&tmV, C::OFF_V, v_full, v_empty, j + 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ------------------------------------------- MMA
      constexpr int fmt = DT<T>::id == TH_BF16 ? 1 : 0;
      constexpr uint32_t id_s = make_idesc_f16(128, C::BN, fmt, 0, 0);
      constexpr uint32_t id_o = make_idesc_f16(128, D, fmt, 0, 1);  // V: MN-major
      const uint32_t qa = smem_u32(sm + C::OFF_Q);
      bool ok = mbar_wait(q_full, 0, abort_flag);
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1, ks = j % NS;
        if (!mbar_wait(&k_full[ks], (j / NS) & 1, abort_flag)) return false;
        if (!mbar_wait(&s_free[s], ((j >> 1) & 1) ^ 1, abort_flag)) return false;
        tc_fence_after();
        const uint32_t ka = smem_u32(sm + C::OFF_K + ks * C::KV_BYTES);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t off = (uint32_t)((k >> 2) * C::BM * 128 + (k & 3) * 32);
          const uint32_t koff = (uint32_t)((k >> 2) * C::BN * 128 + (k & 3) * 32);
          tc_mma_f16(tmem + s * 128, make_desc_sw128(qa + off, 16, 1024), make_desc_sw128(ka + koff, 16, 1024), id_s,
                     k ? 1u : 0u);
        }
        tc_commit(&s_full[s]);
        tc_commit(&k_empty[ks]);
        return true;
      };
      if (ok && nkv > 0) ok = issue_s(0);
      for (int j = 0; ok && j < nkv; ++j) {
        if (j + 1 < nkv && !issue_s(j + 1)) break;
        const int s = j & 1, vs = j % NS;
        if (!mbar_wait(p_full, j & 1, abort_flag) || !mbar_wait(&v_full[vs], (j / NS) & 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t va = smem_u32(sm + C::OFF_V + vs * C::KV_BYTES);
#pragma unroll
        for (int k = 0; k < C::BN / 16; ++k) {
          // A = P_j from TMEM: key half h = k / 4 sits in columns [h*64, h*64+32) of S buffer s, eight
          // columns per 16 keys; B = V kv x D (MN-major, atoms 128 rows apart); half h accumulates into O_h
          const uint32_t pt = tmem + (uint32_t)(s * 128 + (k >> 2) * 64 + (k & 3) * 8);
          tc_mma_f16_ts(tO + (uint32_t)((k >> 2) * D), pt, make_desc_sw128(va + k * 16 * 128, C::BN * 128, 1024),
                        id_o, (j | (k & 3)) ? 1u : 0u);
        }
        tc_commit(&pv_done[s]);
        tc_commit(&s_free[s]);
        tc_commit(&v_empty[vs]);
      }
      tc_commit(mma_done);
    }
  } else {  // ------------------------------------- softmax warps 2..9, two per TMEM lane quarter
    const int q4 = warp & 3;
    const int hh = (warp - 2) >> 2;        // key half of S this warp owns (and its accumulator O_hh)
    const int r = q4 * 32 + lane;          // row within the tile (TMEM lane)
    const int qi = q0 + r;                 // query position
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const float sl2 = p.scale * 1.4426950408889634f;
    constexpr int HB = C::BN / 2, HD = D / 2;
    float* red = reinterpret_cast<float*>(sm + C::OFF_RED);  // [2 halves][128 rows], epilogue only
    const uint32_t tOh = tO + lane_off + (uint32_t)(hh * D);  // this half's accumulator row
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const int s = j & 1;
      ok = __all_sync(0xffffffffu, ok && mbar_wait(&s_full[s], (j >> 1) & 1, abort_flag));
      const int k0 = j * C::BN + hh * HB;  // first key of this warp's columns
      const bool diag = p.causal && (j * C::BN + C::BN - 1 > q0);
      float v[HB];
      float mx = -INFINITY;
      if (ok) {
        tc_fence_after();
        const uint32_t sb = tmem + lane_off + s * 128 + hh * HB;
        uint32_t raw[HB / 32][32];
#pragma unroll
        for (int c = 0; c < HB / 32; ++c) tmem_ld32_issue(sb + c * 32, raw[c]);
#pragma unroll
        for (int c = 0; c < HB / 32; ++c) {
          tmem_wait_ld32(raw[c]);
#pragma unroll
          for (int e = 0; e < 32; ++e) v[c * 32 + e] = __uint_as_float(raw[c][e]);
        }
        tc_fence_before();
        if (diag || k0 + HB > p.seq) {  // masking only in the diagonal block and past the sequence end
#pragma unroll
          for (int e = 0; e < HB; ++e) {
            const int kj = k0 + e;
            if (kj >= p.seq || (diag && kj > qi)) v[e] = -INFINITY;
          }
        }
        float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};  // four independent chains
#pragma unroll
        for (int e = 0; e < HB; ++e) m4[e & 3] = fmaxf(m4[e & 3], v[e]);
        mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * sl2;  // the scale is positive
      }
      const float m_new = fmaxf(m_ref, mx);
      const bool rescale = j > 0 && m_new > m_ref + 8.0f;
      const bool any_rescale = __any_sync(0xffffffffu, rescale);
      // O is rescaled only once O += P_{j-1} V_{j-1} is complete (P_j goes into S_j's own buffer,
      // which nothing else reads before P_j V_j)
      if (j > 0 && any_rescale)
        ok = __all_sync(0xffffffffu, ok && mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, abort_flag));
      if (ok) {
        tc_fence_after();
        if (j == 0) {
          m_ref = m_new;
        } else if (any_rescale) {
          const float f = rescale ? ex2_fast(m_ref - m_new) : 1.f;
          for (int c = 0; c < D; c += 32) {
            float o[32];
            tmem_ld32(tOh + c, o);
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] *= f;
            tmem_st32(tOh + c, o);
          }
          if (rescale) {
            l *= f;
            m_ref = m_new;
          }
        }
        const float mref = (m_ref == -INFINITY) ? 0.f : m_ref;  // fully masked row: P = 0
        // P = exp2(s*scale - m_ref) as 16-bit pairs into TMEM, running sum (2^-inf = 0 for masked scores)
        float pk[HB / 2];
        float l4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < HB / 2; ++c) {
          const float p0 = ex2_fast(fmaf(v[2 * c], sl2, -mref));
          const float p1 = ex2_fast(fmaf(v[2 * c + 1], sl2, -mref));
          l4[(2 * c) & 3] += p0;
          l4[(2 * c + 1) & 3] += p1;
          pk[c] = __uint_as_float(pack2<T>(p0, p1));
        }
        tmem_st32(tmem + lane_off + (uint32_t)(s * 128 + hh * HB), pk);
        l += (l4[0] + l4[1]) + (l4[2] + l4[3]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    // epilogue: O = (O_0 2^(m_0-m) + O_1 2^(m_1-m)) / (l_0 2^(m_0-m) + l_1 2^(m_1-m)), m = max(m_0, m_1);
    // the two warps of a TMEM lane quarter swap (m, l) through a 64-thread barrier of their own
    if (ok && nkv > 0) {
      ok = __all_sync(0xffffffffu, mbar_wait(&pv_done[(nkv - 1) & 1], ((nkv - 1) >> 1) & 1, abort_flag));
      tc_fence_after();
    }
    red[hh * 128 + r] = m_ref;
    named_bar(1 + q4, 64);
    const float m_o = red[(1 - hh) * 128 + r];
    named_bar(1 + q4, 64);
    red[hh * 128 + r] = l;
    named_bar(1 + q4, 64);
    const float l_o = red[(1 - hh) * 128 + r];
    const float m_all = fmaxf(m_ref, m_o);
    const float a_s = m_ref == -INFINITY ? 0.f : ex2_fast(m_ref - m_all);  // this half's weight
    const float a_o = m_o == -INFINITY ? 0.f : ex2_fast(m_o - m_all);      // the other half's
    const float lt = l * a_s + l_o * a_o;
    if (ok) {
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      const float w_s = a_s * inv, w_o = a_o * inv;
      const uint32_t tOo = tO + lane_off + (uint32_t)((1 - hh) * D);
      T* orow = reinterpret_cast<T*>(p.o) + (row0 + qi) * p.ldo + (int64_t)h * D;
      for (int c = hh * HD; c < hh * HD + HD; c += 32) {
        float o[32], o2[32];
        tmem_ld32(tOh + c, o);
        tmem_ld32(tOo + c, o2);
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] = o[e] * w_s + o2[e] * w_o;
        if (qi < p.seq) {
#pragma unroll
          for (int e8 = 0; e8 < 32; e8 += 8) store8<T>(orow + c + e8, o + e8);
        }
      }
    }
  }
  __syncwarp();
  if (threadIdx.x == 64) {  // TMEM must be idle before it is freed
    volatile int dummy = 0;
    mbar_wait(mma_done, 0, &dummy);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// bf16/fp16, head_dim 64/128, 16-byte aligned rows; returns 1 (not taken) otherwise.
template <typename T>
static int attention_tc_try(const th_attention_args* a, cudaStream_t st, int* rc) {
  const int D = a->head_dim;
  if (D != 64 && D != 128) return 1;
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->o) || a->ldq % 8 || a->ldk % 8 ||
      a->ldv % 8 || a->ldo % 8)
    return 1;
  const int64_t T_ = (int64_t)a->batch * a->seq;
  if (T_ >= INT32_MAX) return 1;
  CUtensorMap tq, tk, tv;
  int r = make_tmap_2d(&tq, a->q, a->dtype, (uint64_t)a->hq * D, (uint64_t)T_, (uint64_t)a->ldq * 2, 64, 128, true);
  if (!r) r = make_tmap_2d(&tk, a->k, a->dtype, (uint64_t)a->hkv * D, (uint64_t)T_, (uint64_t)a->ldk * 2, 64, 128, true);
  if (!r) r = make_tmap_2d(&tv, a->v, a->dtype, (uint64_t)a->hkv * D, (uint64_t)T_, (uint64_t)a->ldv * 2, 64, 128, true);
  if (r) { *rc = r; return 0; }
  dim3 grid((unsigned)((a->seq + 127) / 128), (unsigned)a->hq, (unsigned)a->batch);
  if (D == 128) {
    if ((*rc = smem_limit(attention_tc_kernel<T, 128>, AtCfg<128>::SMEM, "th_attention(tcgen05)"))) return 0;
    launch_pdl(attention_tc_kernel<T, 128>, grid, dim3(320), AtCfg<128>::SMEM, st, tq, tk, tv, *a);
  } else {
    if ((*rc = smem_limit(attention_tc_kernel<T, 64>, AtCfg<64>::SMEM, "th_attention(tcgen05)"))) return 0;
    launch_pdl(attention_tc_kernel<T, 64>, grid, dim3(320), AtCfg<64>::SMEM, st, tq, tk, tv, *a);
  }
  *rc = check_launch("th_attention(tcgen05)");
  return 0;
}

}  // namespace th
