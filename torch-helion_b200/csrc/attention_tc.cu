// tcgen05 flash attention (forward) for bf16/fp16, head_dim 64 or 128, in two
// kernels: attention_tc2q_kernel (two 128-row query tiles per CTA, ping-pong on
// the tensor core; the default, described above its definition) and
// attention_tc_kernel below (one tile per CTA; TH_ATTN_TILES=1).
//
// attention_tc_kernel: one CTA = 128 query rows of one (batch, query head); KV blocks of 128 rows.
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

// ---------------------------------------------------------------------------
// attention_tc2q_kernel: two 128-row query tiles per CTA share every K/V
// block, so the tensor core works on one tile while the other tile's softmax
// runs (ping-pong).  320 threads:
//   warp 0     TMA: both query tiles once, then K_i and V_i (K and V rings)
//   warp 1     MMA, issued in the order
//                S0(i) = Q0 K_i^T, O1 += P1(i-1) V(i-1), S1(i) = Q1 K_i^T, O0 += P0(i) V(i)
//              (each product in two halves: keys 64-127 once the softmax has signalled
//              that half of P, then keys 0-63)
//              so that while softmax 0 works on S0(i) the tensor core runs tile 1's
//              product and score block, and the other way round.  P_t(i) lives in
//              the last 64 columns of its S_t buffer (bf16 pairs) and is read by
//              the P.V MMA from TMEM; S_t(i+1) is issued after O_t += P_t(i) V(i)
//              by the same thread, and the tcgen05.mma operations of one thread
//              run in issue order, so the product has read P_t(i) before S_t(i+1)
//              overwrites it.
//   warps 2-5  softmax of tile 0, warps 6-9 of tile 1 (warp w serves TMEM lane
//              quadrant w % 4, so each tile covers all four): one thread per query
//              row (its TMEM lane); online softmax in the log2 domain with a lazy
//              rescale of O_t (only when the running max grows by more than 2^8).
//              O_t is idle while the softmax of block i runs: O_t += P_t(i-1) V(i-1)
//              was issued before S_t(i), and the commit that signalled S_t(i)
//              covers every earlier MMA of the issuing thread.  After the last
//              block the same threads normalise O_t and store it.
// Causal masking: tile 0 stops one KV block before tile 1 (that block lies wholly
// above its diagonal); diagonal blocks are masked per element.
// TMEM: S0 [0,128), S1 [128,256), O0 [256, 256+D), O1 [256+D, 256+2D).
template <int D>
struct At2Cfg {
  static constexpr int BM = 128, BN = 128;
  static constexpr int DA = D / 64;
  static constexpr int Q_BYTES = BM * D * 2;  // one query tile
  static constexpr int KV_BYTES = BN * D * 2;
  // K and V ring depths; at D = 64 the deeper K ring also keeps one CTA per SM (each takes all of TMEM)
  static constexpr int KS = D == 64 ? 3 : 2, VS = 3;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = 2 * Q_BYTES;
  static constexpr int OFF_V = OFF_K + KS * KV_BYTES;
  static constexpr int OFF_BAR = OFF_V + VS * KV_BYTES;
  static constexpr int SMEM = 1024 + OFF_BAR + 256;
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  static_assert(SMEM > 227 * 1024 / 2, "one CTA per SM");
};

template <typename T, int D, int EMU>
__global__ void __launch_bounds__(320, 1)
    attention_tc2q_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, th_attention_args p) {
  using C = At2Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_align<1024>(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;           // [KS]
  uint64_t* k_empty = k_full + C::KS;    // [KS]
  uint64_t* v_full = k_empty + C::KS;    // [VS]
  uint64_t* v_empty = v_full + C::VS;    // [VS]
  uint64_t* s_full = v_empty + C::VS;    // [2] per tile
  uint64_t* p_full = s_full + 2;         // [2] per tile (its 4 softmax warps arrive): all of P
  uint64_t* p_half = p_full + 2;         // [2] per tile: P of keys 64-127 (and O_t rescaled)
  uint64_t* o_done = p_half + 2;         // [2] per tile: its last P.V product is complete
  uint64_t* mma_done = o_done + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqb = (p.seq + 2 * C::BM - 1) / (2 * C::BM);
  const int qb = nqb - 1 - (int)blockIdx.x;  // heaviest (most KV blocks) first when causal
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.hq / p.hkv);
  const int q0 = qb * 2 * C::BM;
  const int64_t row0 = (int64_t)b * p.seq;
  const int nkv_all = (p.seq + C::BN - 1) / C::BN;
  // KV blocks of each tile (the causal bound of its last row)
  const int nkv0 = p.causal ? min(nkv_all, (q0 + C::BM - 1) / C::BN + 1) : nkv_all;
  const int nkv1 = p.causal ? min(nkv_all, (q0 + 2 * C::BM - 1) / C::BN + 1) : nkv_all;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < C::KS; ++s) { mbar_init(&k_full[s], 1); mbar_init(&k_empty[s], 1); }
    for (int s = 0; s < C::VS; ++s) { mbar_init(&v_full[s], 1); mbar_init(&v_empty[s], 1); }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 4);
      mbar_init(&p_half[t], 4);
      mbar_init(&o_done[t], 1);
    }
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
      mbar_arrive_expect_tx(q_full, 2 * C::Q_BYTES);
      for (int t = 0; t < 2; ++t)
        for (int a = 0; a < C::DA; ++a)
          tma_load_2d(sm + C::OFF_Q + t * C::Q_BYTES + a * C::BM * 128, &tmQ, q_full, h * D + a * 64,
                      (int)(row0 + q0 + t * C::BM));
      for (int i = 0; i < nkv1; ++i) {
        const int ks = i % C::KS, vs = i % C::VS;
        if (!mbar_wait(&k_empty[ks], ((i / C::KS) & 1) ^ 1, abort_flag)) break;
        mbar_arrive_expect_tx(&k_full[ks], C::KV_BYTES);
        for (int a = 0; a < C::DA; ++a)
          tma_load_2d(sm + C::OFF_K + ks * C::KV_BYTES + a * C::BN * 128, &tmK, &k_full[ks], hk * D + a * 64,
                      (int)(row0 + i * C::BN));
        if (!mbar_wait(&v_empty[vs], ((i / C::VS) & 1) ^ 1, abort_flag)) break;
        mbar_arrive_expect_tx(&v_full[vs], C::KV_BYTES);
        for (int a = 0; a < C::DA; ++a)
          tma_load_2d(sm + C::OFF_V + vs * C::KV_BYTES + a * C::BN * 128, &tmV, &v_full[vs], hk * D + a * 64,
                      (int)(row0 + i * C::BN));
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ------------------------------------------- MMA
      constexpr int fmt = DT<T>::id == TH_BF16 ? 1 : 0;
      constexpr uint32_t id_s = make_idesc_f16(128, C::BN, fmt, 0, 0);
      constexpr uint32_t id_o = make_idesc_f16(128, D, fmt, 0, 1);  // V: MN-major
      auto issue_s = [&](int t, int i) {  // S_t = Q_t K_i^T
        const uint32_t qa = smem_u32(sm + C::OFF_Q + t * C::Q_BYTES);
        const uint32_t ka = smem_u32(sm + C::OFF_K + (i % C::KS) * C::KV_BYTES);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t off = (uint32_t)((k >> 2) * C::BM * 128 + (k & 3) * 32);
          const uint32_t koff = (uint32_t)((k >> 2) * C::BN * 128 + (k & 3) * 32);
          tc_mma_f16(tmem + t * 128, make_desc_sw128(qa + off, 16, 1024), make_desc_sw128(ka + koff, 16, 1024), id_s,
                     k ? 1u : 0u);
        }
        tc_commit(&s_full[t]);
      };
      // O_t += P_t V_i; keys 2c, 2c+1 of P_t in column 64 + c of S_t.  Keys 64-127 go first, as soon
      // as the softmax has signalled that half, then keys 0-63 (the first product issued for a
      // tile starts the accumulator)
      auto issue_pv = [&](int t, int i) -> bool {
        const uint32_t va = smem_u32(sm + C::OFF_V + (i % C::VS) * C::KV_BYTES);
        if (!mbar_wait(&p_half[t], i & 1, abort_flag)) return false;
        tc_fence_after();
#pragma unroll
        for (int k = 4; k < 8; ++k)
          tc_mma_f16_ts(tO + (uint32_t)(t * D), tmem + (uint32_t)(t * 128 + 64 + k * 8),
                        make_desc_sw128(va + k * 16 * 128, C::BN * 128, 1024), id_o, (i > 0 || k > 4) ? 1u : 0u);
        if (!mbar_wait(&p_full[t], i & 1, abort_flag)) return false;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc_mma_f16_ts(tO + (uint32_t)(t * D), tmem + (uint32_t)(t * 128 + 64 + k * 8),
                        make_desc_sw128(va + k * 16 * 128, C::BN * 128, 1024), id_o, 1u);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, abort_flag);
      for (int i = 0; ok && i < nkv1; ++i) {
        if (!(ok = mbar_wait(&k_full[i % C::KS], (i / C::KS) & 1, abort_flag))) break;
        tc_fence_after();
        if (i < nkv0) issue_s(0, i);
        if (i > 0) {  // tile 1's product of the previous block, then its scores of this one
          if (!(ok = issue_pv(1, i - 1))) break;
          tc_commit(&v_empty[(i - 1) % C::VS]);  // tile 1 is the last reader of V_{i-1}
        }
        issue_s(1, i);
        tc_commit(&k_empty[i % C::KS]);  // ... and of K_i
        if (i < nkv0) {
          if (!(ok = mbar_wait(&v_full[i % C::VS], (i / C::VS) & 1, abort_flag) && issue_pv(0, i))) break;
          if (i == nkv0 - 1) tc_commit(&o_done[0]);
        }
      }
      if (ok) {  // tile 1's last product (its V was not waited for when tile 0 stopped a block early)
        const int i = nkv1 - 1;
        ok = (i < nkv0 || mbar_wait(&v_full[i % C::VS], (i / C::VS) & 1, abort_flag)) && issue_pv(1, i);
        if (ok) {
          tc_commit(&v_empty[i % C::VS]);
          tc_commit(&o_done[1]);
        }
      }
      tc_commit(mma_done);
    }
  } else {  // ---------------------------------------------- softmax + epilogue, one thread per row
    const int t = (warp - 2) >> 2;       // query tile
    const int q4 = warp & 3;             // TMEM lane quadrant
    const int r = q4 * 32 + lane;        // row within the tile (TMEM lane)
    const int qt = q0 + t * C::BM;       // first query of the tile
    const int qi = qt + r;               // this row's query position
    const int nkv = t ? nkv1 : nkv0;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const uint32_t tS = tmem + lane_off + (uint32_t)(t * 128);  // S_t / P_t row
    const uint32_t tOr = tO + lane_off + (uint32_t)(t * D);       // O_t row
    const float sl2 = p.scale * 1.4426950408889634f;
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      ok = __all_sync(0xffffffffu, ok && mbar_wait(&s_full[t], j & 1, abort_flag));
      if (ok) {
        tc_fence_after();
        // Two passes over the 128 scores: all four key chunks loaded for the max, chunks 2-3 kept,
        // then P of chunks 2, 3 and of 0, 1 read again from TMEM (in a diagonal or ragged block,
        // masked before they were stored back).  P of key chunk c goes to columns 64 + 16c, over the scores of chunks
        // 2-3, which are in registers by then; chunks 0-1 are never overwritten.
        const int k0 = j * C::BN;
        const bool edge = (p.causal && k0 + C::BN - 1 > qt) || k0 + C::BN > p.seq;  // diagonal or ragged
        // keys k0 + e with e >= nvalid are masked: past the sequence, or after this row when causal
        const int nvalid = min(p.seq, p.causal ? qi + 1 : p.seq) - k0;
        auto mask = [&](uint32_t(&v)[32], int c) {
          if (edge) {
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (c * 32 + e >= nvalid) v[e] = __float_as_uint(-INFINITY);
          }
        };
        float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        auto vmax = [&](const uint32_t(&v)[32]) {
#pragma unroll
          for (int e = 0; e < 32; ++e) m4[e & 3] = fmaxf(m4[e & 3], __uint_as_float(v[e]));
        };
        uint32_t r0[32], r1[32], r2[32], r3[32];
        tmem_ld32_issue(tS, r0);
        tmem_ld32_issue(tS + 32, r1);
        tmem_ld32_issue(tS + 64, r2);
        tmem_ld32_issue(tS + 96, r3);
        tmem_wait_ld32(r0);
        tmem_wait_ld32(r1);
        if (edge) {  // masked scores of chunks 0-1 go back to TMEM, so their second read needs no mask
          mask(r0, 0);
          mask(r1, 1);
          tmem_st32_nowait(tS, r0);
          tmem_st32_nowait(tS + 32, r1);
        }
        vmax(r0);
        vmax(r1);
        tmem_wait_ld32(r2);
        tmem_wait_ld32(r3);
        mask(r2, 2);
        mask(r3, 3);
        vmax(r2);
        vmax(r3);
        const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * sl2;  // the scale is positive
        // the reference max moves only when the row max grows by more than 2^8 (lazy rescale)
        const float m_new = fmaxf(m_ref, mx);
        const bool rescale = j > 0 && m_new > m_ref + 8.0f;
        const float m_use = (j == 0 || rescale) ? m_new : m_ref;
        const float mref = (m_use == -INFINITY) ? 0.f : m_use;  // fully masked row: P = 0
        const uint64_t sl2p = f2_pack(sl2, sl2), nmp = f2_pack(-mref, -mref);
        uint64_t lp[2] = {0ull, 0ull};  // packed partial row sums (0ull is +0.0f, +0.0f)
        // exp2 (EMU of every 16 pairs on the FMA pipe, the rest on the special-function unit),
        // row sum, bf16 pairs to P columns 64 + 16c
        auto emit = [&](const uint32_t(&v)[32], int c) {
          uint32_t pk[16];
#pragma unroll
          for (int w = 0; w < 16; ++w) {
            float a0, a1, p0, p1;
            f2_unpack(f2_fma(f2_pack(__uint_as_float(v[2 * w]), __uint_as_float(v[2 * w + 1])), sl2p, nmp), a0, a1);
            if (EMU > 0 && (w * EMU) % 16 < EMU) {
              ex2_poly2(a0, a1, p0, p1);
            } else {
              p0 = ex2_fast(a0);
              p1 = ex2_fast(a1);
            }
            lp[w & 1] = f2_add(lp[w & 1], f2_pack(p0, p1));
            pk[w] = pack2<T>(p0, p1);
          }
          tmem_st16_nowait(tS + 64 + c * 16, pk);
        };
        if (edge) tmem_wait_st();  // the masked chunks 0-1 are in TMEM before they are read again
        emit(r2, 2);
        tmem_ld32_issue(tS, r0);  // chunk 0 again, while chunk 3 becomes P
        emit(r3, 3);
        // O_t is idle (see above) until this block's first half of P is signalled: rescale it in place
        const float f = rescale ? ex2_fast(m_ref - m_new) : 1.f;
        if (__any_sync(0xffffffffu, rescale)) {
          for (int c = 0; c < D; c += 16) {
            uint32_t o[16];
            tmem_ld16_issue(tOr + c, o);
            tmem_wait_ld(o);
#pragma unroll
            for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
            tmem_st16_nowait(tOr + c, o);
          }
        }
        tmem_wait_st();  // P of keys 64-127 (and O_t) in TMEM: the product may start on that half
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_half[t]);
        tmem_wait_ld32(r0);
        tmem_ld32_issue(tS + 32, r1);
        emit(r0, 0);
        tmem_wait_ld32(r1);
        emit(r1, 1);
        tmem_wait_st();
        float l0, l1, l2, l3;
        f2_unpack(lp[0], l0, l1);
        f2_unpack(lp[1], l2, l3);
        l = fmaf(l, f, (l0 + l1) + (l2 + l3));
        m_ref = m_use;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (!ok) mbar_arrive(&p_half[t]);  // (sent mid-block when the block ran)
        mbar_arrive(&p_full[t]);
      }
    }
    // epilogue: O_t / l once the tile's last product is complete
    if (ok) {
      ok = __all_sync(0xffffffffu, mbar_wait(&o_done[t], 0, abort_flag));
      tc_fence_after();
    }
    if (ok) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      T* orow = reinterpret_cast<T*>(p.o) + (row0 + qi) * p.ldo + (int64_t)h * D;
      for (int c = 0; c < D; c += 32) {
        float o[32];
        tmem_ld32(tOr + c, o);
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] *= inv;
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

// TH_ATTN_TILES=1 selects the one-tile kernel (default: two tiles per CTA)
static bool attn_two_tiles() {
  static const bool v = [] {
    const char* e = getenv("TH_ATTN_TILES");
    return !(e && e[0] == '1');
  }();
  return v;
}

// How many of every 16 exponential pairs of the two-tile kernel run on the FMA pipe: TH_ATTN_EMU=0|4|8,
// default 4 (C3 attention, B8 S4096 causal: 1166 / 1141 / 1147 us for 0 / 4 / 8)
static int attn_emu() {
  static const int v = [] {
    const char* e = getenv("TH_ATTN_EMU");
    return e ? atoi(e) : 4;
  }();
  return v;
}

template <typename T, int D, int EMU>
static int attention_tc2q_launch(dim3 grid, cudaStream_t st, const CUtensorMap& tq, const CUtensorMap& tk,
                                 const CUtensorMap& tv, const th_attention_args* a) {
  if (int rc = smem_limit(attention_tc2q_kernel<T, D, EMU>, At2Cfg<D>::SMEM, "th_attention(tcgen05, 2 tiles)"))
    return rc;
  launch_pdl(attention_tc2q_kernel<T, D, EMU>, grid, dim3(320), At2Cfg<D>::SMEM, st, tq, tk, tv, *a);
  return check_launch("th_attention(tcgen05, 2 tiles)");
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
  if (attn_two_tiles()) {
    const dim3 grid2((unsigned)((a->seq + 255) / 256), (unsigned)a->hq, (unsigned)a->batch);
    const int emu = attn_emu();
    if (D == 128) {
      if (emu == 4) *rc = attention_tc2q_launch<T, 128, 4>(grid2, st, tq, tk, tv, a);
      else if (emu == 8) *rc = attention_tc2q_launch<T, 128, 8>(grid2, st, tq, tk, tv, a);
      else *rc = attention_tc2q_launch<T, 128, 0>(grid2, st, tq, tk, tv, a);
    } else {
      if (emu == 4) *rc = attention_tc2q_launch<T, 64, 4>(grid2, st, tq, tk, tv, a);
      else if (emu == 8) *rc = attention_tc2q_launch<T, 64, 8>(grid2, st, tq, tk, tv, a);
      else *rc = attention_tc2q_launch<T, 64, 0>(grid2, st, tq, tk, tv, a);
    }
    return 0;
  }
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
