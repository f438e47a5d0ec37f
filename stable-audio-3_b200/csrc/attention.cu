// Sliding-window (and full / cross) attention on tcgen05 for sm_100a.
//
// Replaces the windowed flash-attention call of Attention.apply_attn
// (stable_audio_3/models/transformer.py:620-666, window_size=(wl, wr)) and its
// math-equivalent fallbacks (_sliding_window_chunked_halo_sdpa :143-159,
// _sliding_window_additive_mask :118-127), plus the differential combine
// out - out_diff of Attention.forward (:790-795): both softmax passes run in
// the same CTA and share the V tiles.
//
// One CTA = 128 query rows of one head of one sequence, 128 threads (thread i
// owns query row i: its S row and O row live in TMEM lane i).
//   * The key range is clipped to the window of the tile's queries
//     ([i0 - wl, i1 + wr] intersected with the sequence), so key tiles that are
//     fully masked are never loaded or multiplied; the two edge tiles are
//     masked element-wise.
//   * Thread 0 issues TMA and the tcgen05.mma ops: S = Q K^T (M=128, N=128,
//     K=64) into TMEM columns [0,128); O_tile = P V (M=128, N=64, K=128) into
//     columns [128,192). Q is loaded once per pass, K tiles are double-buffered
//     (tile t+1 loads during tile t), and the single V buffer is refilled as
//     soon as P V of the previous tile retires, overlapping the next S MMA and
//     softmax. Shared memory: Q 16 KB + K 2x16 KB + V 16 KB + P 32 KB = 96 KB,
//     so two CTAs (2 x 256 TMEM columns) share an SM.
//   * Softmax is online in fp32 (exp2 domain). P is written to shared memory
//     as bf16 in the 128-byte-swizzled K-major layout the MMA reads; V is used
//     MN-major straight from its TMA tile.
#include "common.cuh"
#include "host_util.h"

namespace sa3 {
SA3_DEFINE_ERROR_READER(read_error_attention)

constexpr int ATT_BM = 128;
constexpr int ATT_BN = 128;
constexpr int ATT_TILE_BYTES = 128 * 128;  // 128 rows x 64 bf16
constexpr int ATT_SMEM = ATT_TILE_BYTES * (1 + 2 + 1 + 2) + 1024 + 256;
constexpr int ATT_TMEM_COLS = 256;

struct AttnParams {
  int f16;  // 1: fp16 operands / output, 0: bf16
  const int* cu_q;
  const int* cu_k;
  int Lq, Lk;  // uniform lengths when cu_q / cu_k are NULL
  int heads;
  int wl, wr;
  float scale_log2;
  int npass;
  void* out;
  long long ldo;
  float* amax_out;
};

__device__ __forceinline__ uint32_t pack_2(float lo, float hi, bool f16) {
  if (f16) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  return pack_bf16x2(lo, hi);
}

__device__ __forceinline__ void att_issue(const CUtensorMap* tm, uint8_t* dst, uint64_t* bar, int col, int row) {
  mbar_arrive_expect_tx(bar, ATT_TILE_BYTES);
  tma_load_2d(dst, tm, bar, col, row);
}

__global__ void __launch_bounds__(128, 2)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmQ2,
                        const __grid_constant__ CUtensorMap tmK2, const __grid_constant__ CUtensorMap tmV2,
                        AttnParams p) {
  const int t = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int qs = p.cu_q ? __ldg(p.cu_q + b) : b * p.Lq;
  const int lq = p.cu_q ? __ldg(p.cu_q + b + 1) - qs : p.Lq;
  const int ks = p.cu_k ? __ldg(p.cu_k + b) : b * p.Lk;
  const int lk = p.cu_k ? __ldg(p.cu_k + b + 1) - ks : p.Lk;
  const int i0 = t * ATT_BM;
  if (i0 >= lq) return;  // uniform per CTA, before any barrier / TMEM use
  const int i_last = min(i0 + ATT_BM, lq) - 1;
  const int dlt = lk - lq;
  const int j_lo = p.wl < 0 ? 0 : max(0, i0 + dlt - p.wl);
  const int j_hi = p.wr < 0 ? lk : min(lk, i_last + dlt + p.wr + 1);
  const int ntiles = j_hi > j_lo ? (j_hi - j_lo + ATT_BN - 1) / ATT_BN : 0;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  // K tiles at smem + (1 + buf) * TILE.
#define SK(bf) (smem + (1 + (bf)) * ATT_TILE_BYTES)
  uint8_t* sV = smem + 3 * ATT_TILE_BYTES;
  uint8_t* sP = smem + 4 * ATT_TILE_BYTES;  // two 16 KB K-major sub-tiles (kv 0..63, 64..127)
  uint64_t* bar_q = reinterpret_cast<uint64_t*>(smem + 6 * ATT_TILE_BYTES);
  uint64_t* bar_kv = bar_q + 1;  // [2]: K tiles
  uint64_t* bar_s = bar_q + 3;
  uint64_t* bar_o = bar_q + 4;
  uint64_t* bar_v = bar_q + 5;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_q + 6);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5;
  if (tid == 0) {
    mbar_init(bar_q, 1);
    mbar_init(&bar_kv[0], 1);
    mbar_init(&bar_kv[1], 1);
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
    mbar_init(bar_v, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    if (p.npass > 1) {
      tma_prefetch_desc(&tmQ2);
      tma_prefetch_desc(&tmK2);
      tma_prefetch_desc(&tmV2);
    }
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, ATT_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s = tmem + ((uint32_t)(warp * 32) << 16);  // this warp's lanes, S columns
  const uint32_t t_o = t_s + 128;                              // O columns

  const int col = h * 64;
  const int i = i0 + tid;  // this thread's query row (sequence coordinate)
  const float NEG_INF = -INFINITY;

  const int fmt = p.f16 ? 0 : 1;  // kind::f16 operand format: 0 = f16, 1 = bf16
  const uint32_t idesc_s = make_idesc(128, 128, fmt, fmt, 0, 0);
  const uint32_t idesc_o = make_idesc(128, 64, fmt, fmt, 0, 1);

  float o_prev[64];
  float o[64];
#pragma unroll
  for (int d = 0; d < 64; ++d) o_prev[d] = 0.f;

  uint32_t q_phase = 0;
  int gidx = 0;  // global K/V tile counter across passes (buffer = gidx & 1)
  int kv_issued0 = 0, kv_issued1 = 0, v_issued = 0;
  bool bad = false;

  for (int pass = 0; pass < p.npass; ++pass) {
    const CUtensorMap* tq = pass ? &tmQ2 : &tmQ;
    const CUtensorMap* tk = pass ? &tmK2 : &tmK;
    const CUtensorMap* tv = pass ? &tmV2 : &tmV;
    float m_i = NEG_INF, l_i = 0.f;
#pragma unroll
    for (int d = 0; d < 64; ++d) o[d] = 0.f;

    if (tid == 0 && ntiles > 0 && !*abort_flag) {
      mbar_arrive_expect_tx(bar_q, ATT_TILE_BYTES);
      tma_load_2d(sQ, tq, bar_q, col, qs + i0);
      const int bf = gidx & 1;
      att_issue(tk, SK(bf), &bar_kv[bf], col, ks + j_lo);
      if (bf) ++kv_issued1; else ++kv_issued0;
      att_issue(tv, sV, bar_v, col, ks + j_lo);  // previous P V retired (bar_o waited)
      ++v_issued;
    }

    for (int it = 0; it < ntiles; ++it, ++gidx) {
      const int bf = gidx & 1;
      const uint32_t ph = (uint32_t)(gidx >> 1) & 1;
      const int j0 = j_lo + it * ATT_BN;
      if (tid == 0) {
        if (it + 1 < ntiles && !*abort_flag) {
          const int nb = (gidx + 1) & 1;
          att_issue(tk, SK(nb), &bar_kv[nb], col, ks + j0 + ATT_BN);
          if (nb) ++kv_issued1; else ++kv_issued0;
        }
        bool ok = true;
        if (it == 0) ok = mbar_wait(bar_q, q_phase, abort_flag, 20);
        ok = ok && mbar_wait(&bar_kv[bf], ph, abort_flag, 21);
        if (ok) {
          tc_fence_after();
          const uint64_t qd = sdesc_kmajor_sw128(smem_u32(sQ));
          const uint64_t kd = sdesc_kmajor_sw128(smem_u32(SK(bf)));
#pragma unroll
          for (int k = 0; k < 4; ++k) mma_f16_ss(tmem, qd + 2 * k, kd + 2 * k, idesc_s, k != 0);
        }
        tc_commit(bar_s);
      }
      if (!mbar_wait(bar_s, (uint32_t)gidx & 1, abort_flag, 22)) bad = true;
      tc_fence_after();

      // ---- online softmax over this thread's row of S
      float mx = NEG_INF;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float sv[32];
        tmem_ld32(t_s + c * 32, sv);
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int j = j0 + c * 32 + e;
          const int dj = j - i - dlt;
          const bool valid = (j < j_hi) && (p.wl < 0 || dj >= -p.wl) && (p.wr < 0 || dj <= p.wr);
          mx = valid ? fmaxf(mx, sv[e]) : mx;
        }
      }
      const float m_new = fmaxf(m_i, mx * p.scale_log2);
      const float alpha = (m_new == NEG_INF) ? 1.f : fast_exp2(m_i - m_new);
      const float m_use = (m_new == NEG_INF) ? 0.f : m_new;
      float rowsum = 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float sv[32];
        tmem_ld32(t_s + c * 32, sv);
        float pv[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int j = j0 + c * 32 + e;
          const int dj = j - i - dlt;
          const bool valid = (j < j_hi) && (p.wl < 0 || dj >= -p.wl) && (p.wr < 0 || dj <= p.wr);
          pv[e] = valid ? fast_exp2(sv[e] * p.scale_log2 - m_use) : 0.f;
          rowsum += pv[e];
        }
        // Row `tid` of P: columns c*32.. in sub-tile c/2, 16-byte chunks (c%2)*4 + q.
        uint8_t* rowbase = sP + (c >> 1) * ATT_TILE_BYTES + tid * 128;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int ch = ((c & 1) * 4 + q) ^ (tid & 7);
          uint4 u;
          u.x = pack_2(pv[q * 8 + 0], pv[q * 8 + 1], p.f16);
          u.y = pack_2(pv[q * 8 + 2], pv[q * 8 + 3], p.f16);
          u.z = pack_2(pv[q * 8 + 4], pv[q * 8 + 5], p.f16);
          u.w = pack_2(pv[q * 8 + 6], pv[q * 8 + 7], p.f16);
          *reinterpret_cast<uint4*>(rowbase + ch * 16) = u;
        }
      }
      l_i = l_i * alpha + rowsum;
      m_i = m_new;
#pragma unroll
      for (int d = 0; d < 64; ++d) o[d] *= alpha;

      fence_proxy_async_smem();
      tc_fence_before();
      __syncthreads();
      if (tid == 0) {
        tc_fence_after();
        if (mbar_wait(bar_v, (uint32_t)gidx & 1, abort_flag, 25)) {
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint64_t pd = sdesc_kmajor_sw128(smem_u32(sP + (k >> 2) * ATT_TILE_BYTES)) + 2 * (k & 3);
            const uint64_t vd = sdesc_mnmajor_sw128(smem_u32(sV) + k * 2048, ATT_TILE_BYTES);
            mma_f16_ss(tmem + 128, pd, vd, idesc_o, k != 0);
          }
        }
        tc_commit(bar_o);
      }
      if (!mbar_wait(bar_o, (uint32_t)gidx & 1, abort_flag, 23)) bad = true;
      tc_fence_after();
      if (tid == 0 && it + 1 < ntiles && !*abort_flag) {
        // sV is free once P V of this tile retired: refill it for the next tile.
        att_issue(tv, sV, bar_v, col, ks + j0 + ATT_BN);
        ++v_issued;
      }
      {
        float ov[32];
        tmem_ld32(t_o, ov);
#pragma unroll
        for (int d = 0; d < 32; ++d) o[d] += ov[d];
        tmem_ld32(t_o + 32, ov);
#pragma unroll
        for (int d = 0; d < 32; ++d) o[32 + d] += ov[d];
      }
      tc_fence_before();
    }
    q_phase ^= 1;
    const float inv_l = l_i > 0.f ? 1.f / l_i : 0.f;
    if (pass == 0) {
#pragma unroll
      for (int d = 0; d < 64; ++d) o_prev[d] = o[d] * inv_l;
    } else {
#pragma unroll
      for (int d = 0; d < 64; ++d) o_prev[d] -= o[d] * inv_l;
    }
    // Every thread must be done with sQ before thread 0 reloads it for the next pass.
    __syncthreads();
  }

  // ---- store (row-major token rows, this head's 64 columns)
  float amax = 0.f;
  if (i <= i_last && !bad && !*abort_flag) {
    uint16_t* dst = reinterpret_cast<uint16_t*>(p.out) + (long long)(qs + i) * p.ldo + col;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      uint4 u;
      u.x = pack_2(o_prev[q * 8 + 0], o_prev[q * 8 + 1], p.f16);
      u.y = pack_2(o_prev[q * 8 + 2], o_prev[q * 8 + 3], p.f16);
      u.z = pack_2(o_prev[q * 8 + 4], o_prev[q * 8 + 5], p.f16);
      u.w = pack_2(o_prev[q * 8 + 6], o_prev[q * 8 + 7], p.f16);
      reinterpret_cast<uint4*>(dst)[q] = u;
    }
    if (p.amax_out) {
#pragma unroll
      for (int d = 0; d < 64; ++d)
        amax = fmaxf(amax, fabsf(p.f16 ? __half2float(__float2half(o_prev[d]))
                                       : __bfloat162float(__float2bfloat16(o_prev[d]))));
    }
  }
  if (p.amax_out) {
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, s));
    if ((tid & 31) == 0) atomic_max_nonneg(p.amax_out, amax);
  }

  // ---- teardown: drain any TMA still in flight after an abort, free TMEM.
  if (tid == 0 && *abort_flag) {
    volatile int never = 0;
    if (kv_issued0 > 0) mbar_wait(&bar_kv[0], (uint32_t)(kv_issued0 - 1) & 1, &never, 24);
    if (kv_issued1 > 0) mbar_wait(&bar_kv[1], (uint32_t)(kv_issued1 - 1) & 1, &never, 24);
    if (v_issued > 0) mbar_wait(bar_v, (uint32_t)(v_issued - 1) & 1, &never, 26);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, ATT_TMEM_COLS);
#undef SK
}

}  // namespace sa3

using namespace sa3;

extern "C" int sa3_attention(const void* q, const void* k, const void* v, const void* q2, const void* k2,
                             const void* v2, void* out,
                             const int* cu_seqlens_q, const int* cu_seqlens_k, int batch, int max_seqlen_q,
                             int max_seqlen_k, int total_q, int total_k, int heads, int head_dim, long long ldq,
                             long long ldk, long long ldv, long long ldo, int window_left, int window_right,
                             float softmax_scale, int dtype, float* amax_out, void* stream) {
  if (!q || !k || !v || !out || batch <= 0 || heads <= 0 || max_seqlen_q <= 0 || max_seqlen_k <= 0)
    return SA3_ERR_ARG;
  if (head_dim != 64) return SA3_ERR_UNSUPPORTED;
  if (dtype != SA3_DT_BF16 && dtype != SA3_DT_F16) return SA3_ERR_DTYPE;
  if ((q2 == nullptr) != (k2 == nullptr)) return SA3_ERR_ARG;
  if (v2 && !q2) return SA3_ERR_ARG;
  if ((cu_seqlens_q == nullptr) != (cu_seqlens_k == nullptr)) return SA3_ERR_ARG;
  if (!cu_seqlens_q) {
    total_q = batch * max_seqlen_q;
    total_k = batch * max_seqlen_k;
  }
  if (total_q <= 0 || total_k <= 0) return SA3_ERR_ARG;
  const long long width = (long long)heads * 64;
  if (ldq < width || ldk < width || ldv < width || ldo < width) return SA3_ERR_ARG;
  if (!aligned16(out) || (ldo % 8)) return SA3_ERR_ALIGN;
  if (batch > 65535 || heads > 65535) return SA3_ERR_UNSUPPORTED;

  CUtensorMap mq, mk, mv, mq2, mk2, mv2;
  const auto dt = dtype == SA3_DT_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  int rc;
  if ((rc = make_tmap_2d(&mq, q, dt, 2, width, total_q, ldq, 64, 128))) return rc;
  if ((rc = make_tmap_2d(&mk, k, dt, 2, width, total_k, ldk, 64, 128))) return rc;
  if ((rc = make_tmap_2d(&mv, v, dt, 2, width, total_k, ldv, 64, 128))) return rc;
  if (q2) {
    if ((rc = make_tmap_2d(&mq2, q2, dt, 2, width, total_q, ldq, 64, 128))) return rc;
    if ((rc = make_tmap_2d(&mk2, k2, dt, 2, width, total_k, ldk, 64, 128))) return rc;
  } else {
    mq2 = mq;
    mk2 = mk;
  }
  if (v2) {
    if ((rc = make_tmap_2d(&mv2, v2, dt, 2, width, total_k, ldv, 64, 128))) return rc;
  } else {
    mv2 = mv;
  }
  AttnParams p;
  p.f16 = dtype == SA3_DT_F16;
  p.cu_q = cu_seqlens_q;
  p.cu_k = cu_seqlens_k;
  p.Lq = max_seqlen_q;
  p.Lk = max_seqlen_k;
  p.heads = heads;
  p.wl = window_left;
  p.wr = window_right;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.npass = q2 ? 2 : 1;
  p.out = out;
  p.ldo = ldo;
  p.amax_out = amax_out;
  dim3 grid((max_seqlen_q + ATT_BM - 1) / ATT_BM, heads, batch);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if ((rc = ensure_smem(attention_tc_kernel, ATT_SMEM))) return rc;
  attention_tc_kernel<<<grid, 128, ATT_SMEM, st>>>(mq, mk, mv, mq2, mk2, mv2, p);
  return launch_status();
}

extern "C" int sa3_diff_attn_swa(const void* q_bat, const void* k_bat, const void* v_bat, void* out, int dtype,
                                 int batch, int seqlen, int num_heads, int head_dim, int window, void* stream) {
  // q/k/v_bat: [B, N, 2H, d] (stream 1 = heads 0..H-1, stream 2 = heads H..2H-1); out: [B, N, H, d].
  if (!q_bat || !k_bat || !v_bat || !out || batch <= 0 || seqlen <= 0 || num_heads <= 0) return SA3_ERR_ARG;
  if (head_dim != 64) return SA3_ERR_UNSUPPORTED;
  const size_t esz = 2;
  const long long hw = (long long)num_heads * head_dim;  // elements of one stream's heads in a row
  const char* q = static_cast<const char*>(q_bat);
  const char* k = static_cast<const char*>(k_bat);
  const char* v = static_cast<const char*>(v_bat);
  return sa3_attention(q, k, v, q + hw * esz, k + hw * esz, v + hw * esz, out, nullptr, nullptr, batch, seqlen,
                       seqlen, batch * seqlen, batch * seqlen, num_heads, head_dim, 2 * hw, 2 * hw, 2 * hw, hw,
                       window, window, 1.0f / sqrtf((float)head_dim), dtype, nullptr, stream);
}
