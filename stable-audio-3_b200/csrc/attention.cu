// Sliding-window (and full / cross) attention on tcgen05 for sm_100a.
//
// Replaces the windowed flash-attention call of Attention.apply_attn
// (stable_audio_3/models/transformer.py:620-666, window_size=(wl, wr)) and its
// math-equivalent fallbacks (_sliding_window_chunked_halo_sdpa :143-159,
// _sliding_window_additive_mask :118-127), plus the differential combine
// out - out_diff of Attention.forward (:790-795).
//
// Persistent: one CTA per SM walks work items (pairs of query tiles, query tile
// fastest, so CTAs that run together share K/V tiles in L2); barrier phases run
// on across items. Unit u of a CTA owns query tile 2 * pair + u (128 rows x one
// head); a differential head runs its two softmax streams as two passes of the
// same unit. 384 threads, warp-specialised:
//   warps 0 / 3 (lane 0)  TMA for unit 0 / 1: Q per pass (two slots), K three
//                    tiles and V two tiles deep, K one tile ahead of V.
//   warps 1 / 2      tcgen05.mma for unit 0 / 1, issued by one elected lane of
//                    the converged warp: S = Q K^T (M=128, N=128, K=64, both
//                    from shared memory) and O (+)= P V (M=128, N=64, K=128, P
//                    from TMEM, V MN-major straight from its TMA tile). Each
//                    unit has its own loader and issuer, so the two units never
//                    wait on each other.
//   warps 4..7, 8..11  softmax warpgroup of unit 0 / unit 1; thread r owns query
//                    row r (TMEM lane r).
// TMEM per unit (256 columns): S [0,128) fp32, P [128,192) as packed 16-bit
// pairs, O [192,256) fp32. The softmax copies a whole S row into registers and
// releases the S columns at once, so the tensor core computes S of the next key
// tile while the exponentials of this one run; P V follows when P is written.
// O stays in TMEM for the whole key range. The online softmax keeps a
// reference maximum per row and only moves it (rescaling O and the row sum)
// when a tile's maximum exceeds it by more than 2^8, which keeps every exp2
// argument <= 8 and leaves the result exactly softmax(S) V. A differential head
// normalises stream 1 at the end of its pass and keeps it in registers as 16-bit
// values (the rounding the reference applies to each attention output before
// out - out_diff), then subtracts stream 2's result from it.
// The key range of a unit is clipped to the window of its queries, so fully
// masked key tiles are never loaded or multiplied; tiles that lie entirely
// inside every row's band skip masking, edge tiles mask with a bit mask.
// Shared memory: per unit Q 2x16 KB + K 3x16 KB + V 2x16 KB = 112 KB.
#include "common.cuh"
#include "host_util.h"

namespace sa3 {
SA3_DEFINE_ERROR_READER(read_error_attention)

constexpr int ATT_BM = 128;
constexpr int ATT_BN = 128;
constexpr int ATT_TILE = 128 * 128;  // 128 rows x 64 16-bit elements
constexpr int ATT_QS = 2, ATT_KS = 3, ATT_VS = 2;         // Q slots, K stages, V stages per unit
constexpr int ATT_UNIT_TILES = ATT_QS + ATT_KS + ATT_VS;  // 7 tiles of 16 KB
constexpr int ATT_THREADS = 384;
constexpr int ATT_SMEM = 2 * ATT_UNIT_TILES * ATT_TILE + 1024 + 1024;  // tiles + alignment slack + barriers
constexpr float ATT_RESCALE_LOG2 = 8.f;  // move the reference maximum only when it grows by more than this
constexpr int ATT_TMEM_COLS = 512;
constexpr int ATT_REGS_LAUNCH = 168;  // per thread at launch: 65536 / 384 rounded down to a multiple of 8
constexpr int ATT_REGS_LOW = 64;      // TMA / MMA warpgroup after the split
constexpr int ATT_REGS_HIGH = 216;    // each softmax warpgroup after the split
static_assert(ATT_REGS_LOW * 128 + ATT_REGS_HIGH * 256 <= ATT_REGS_LAUNCH * ATT_THREADS,
              "register split exceeds the block's launch allocation");

struct AttnParams {
  int f16;  // 1: fp16 operands / output, 0: bf16
  const int* cu_q;
  const int* cu_k;
  int Lq, Lk;  // uniform lengths when cu_q / cu_k are NULL
  int heads;
  int wl, wr;
  float scale_log2;
  int diff;  // differential: unit 1 = second stream of the same rows
  void* out;
  long long ldo;
  float* amax_out;
};

struct Unit {
  int qs, ks, lq, lk, i0, dlt, j_lo, ntiles;
  bool valid;
};

__device__ __forceinline__ Unit make_unit(const AttnParams& p, int b, int tile) {
  Unit u;
  u.qs = p.cu_q ? __ldg(p.cu_q + b) : b * p.Lq;
  u.lq = p.cu_q ? __ldg(p.cu_q + b + 1) - u.qs : p.Lq;
  u.ks = p.cu_k ? __ldg(p.cu_k + b) : b * p.Lk;
  u.lk = p.cu_k ? __ldg(p.cu_k + b + 1) - u.ks : p.Lk;
  u.i0 = tile * ATT_BM;
  u.valid = u.i0 < u.lq;
  u.dlt = u.lk - u.lq;
  u.j_lo = 0;
  u.ntiles = 0;
  if (u.valid) {
    const int i_last = min(u.i0 + ATT_BM, u.lq) - 1;
    u.j_lo = p.wl < 0 ? 0 : max(0, u.i0 + u.dlt - p.wl);
    const int j_hi = p.wr < 0 ? u.lk : min(u.lk, i_last + u.dlt + p.wr + 1);
    u.ntiles = j_hi > u.j_lo ? (j_hi - u.j_lo + ATT_BN - 1) / ATT_BN : 0;
  }
  return u;
}

__device__ __forceinline__ uint32_t pack_2(float lo, float hi, bool f16) {
  if (f16) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  return pack_bf16x2(lo, hi);
}

// Packed pairs of fp32 (sm_100 f32x2 arithmetic: one instruction per two lanes of data).
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 f2_split(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

constexpr uint32_t NEG_INF_BITS = 0xff800000u;

// Edge tile: scores of columns outside [lo, hi) (chunk-relative) become -inf.
__device__ __forceinline__ void mask_chunk(uint32_t (&s)[32], int lo, int hi) {
  const int a = min(max(lo, 0), 32), b = min(max(hi, 0), 32);
  const uint32_t below_b = b >= 32 ? 0xffffffffu : ((1u << b) - 1u);
  const uint32_t below_a = a >= 32 ? 0xffffffffu : ((1u << a) - 1u);
  const uint32_t m = below_b & ~below_a;
#pragma unroll
  for (int e = 0; e < 32; ++e) s[e] = (m >> e) & 1u ? s[e] : NEG_INF_BITS;
}

// Running maxima over one chunk, eight independent chains.
__device__ __forceinline__ void max_chunk(const uint32_t (&s)[32], float (&m)[8]) {
#pragma unroll
  for (int t = 0; t < 8; ++t)
    m[t] = fmax3(fmax3(m[t], __uint_as_float(s[4 * t]), __uint_as_float(s[4 * t + 1])),
                 __uint_as_float(s[4 * t + 2]), __uint_as_float(s[4 * t + 3]));
}

// P = exp2(s * scale - m) for one chunk as packed 16-bit pairs, row sums into four f32x2 chains.
__device__ __forceinline__ void exp_chunk(const uint32_t (&s)[32], uint64_t scale2, uint64_t negm2,
                                          uint64_t (&acc)[4], uint32_t (&w)[16], bool f16) {
#pragma unroll
  for (int e = 0; e < 32; e += 2) {
    const float2 x = f2_split(ffma2(f2(__uint_as_float(s[e]), __uint_as_float(s[e + 1])), scale2, negm2));
    const float p0 = fast_exp2(x.x), p1 = fast_exp2(x.y);
    acc[(e >> 1) & 3] = fadd2(acc[(e >> 1) & 3], f2(p0, p1));
    w[e >> 1] = pack_2(p0, p1, f16);
  }
}

// tcgen05.mma / commit issued by one elected lane of a converged warp, descriptors given as (low
// word, shared high word): the issue loop only adds constants to the low word (the start-address
// field). Running the issue loop on the whole warp keeps its operands warp-uniform, which lets the
// MMAs go out back to back (from a single lane in a divergent branch the 64-wide P V steps issue at
// about 60% of the tensor rate).
__device__ __forceinline__ void mma_ss_lo(uint32_t d_tmem, uint32_t a_lo, uint32_t b_lo, uint32_t hi,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b32 r;\n\t.reg .b64 da, db;\n\t"
      "setp.ne.b32 p, %5, 0;\n\t"
      "mov.b64 da, {%1, %3};\n\t"
      "mov.b64 db, {%2, %3};\n\t"
      "elect.sync r|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %4, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_lo), "r"(b_lo), "r"(hi), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_ts_lo(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_lo, uint32_t b_hi,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b32 r;\n\t.reg .b64 db;\n\t"
      "setp.ne.b32 p, %5, 0;\n\t"
      "mov.b64 db, {%2, %3};\n\t"
      "elect.sync r|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], db, %4, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void commit_elect(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t.reg .b32 r;\n\t"
      "elect.sync r|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}\n" ::"r"(smem_u32(bar))
      : "memory");
}
// mbar_wait on every lane of a converged warp; the warp agrees on the outcome.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int site) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, site));
}

// Work item = (pair of consecutive query tiles, head, sequence), query tile fastest. Unit u of the
// CTA takes query tile 2 * pair + u; a differential head runs its two streams as two passes.
__device__ __forceinline__ void decode_item(const AttnParams& p, int item, int pairs_per_head, int& b, int& h,
                                            int& tile0) {
  const int pair = item % pairs_per_head;
  const int rest = item / pairs_per_head;
  h = rest % p.heads;
  b = rest / p.heads;
  tile0 = 2 * pair;
}

template <bool NARROW>
__global__ void __launch_bounds__(ATT_THREADS, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmQ2,
                        const __grid_constant__ CUtensorMap tmK2, const __grid_constant__ CUtensorMap tmV2,
                        AttnParams p, int num_items, int pairs_per_head) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
#define SQ(u, b) (smem + ((u) * ATT_UNIT_TILES + (b)) * ATT_TILE)
#define SK(u, s) (smem + ((u) * ATT_UNIT_TILES + ATT_QS + (s)) * ATT_TILE)
#define SV(u, s) (smem + ((u) * ATT_UNIT_TILES + ATT_QS + ATT_KS + (s)) * ATT_TILE)
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 2 * ATT_UNIT_TILES * ATT_TILE);
  uint64_t* q_full = bars;          // [unit][ATT_QS]
  uint64_t* q_empty = bars + 4;     // [unit][ATT_QS]
  uint64_t* k_full = bars + 8;      // [unit][ATT_KS]
  uint64_t* k_empty = bars + 14;    // [unit][ATT_KS]
  uint64_t* v_full = bars + 20;     // [unit][ATT_VS]
  uint64_t* v_empty = bars + 24;    // [unit][ATT_VS]
  uint64_t* s_full = bars + 28;     // [unit]  S of a tile is in TMEM
  uint64_t* s_empty = bars + 30;    // [unit]  the softmax holds it in registers (4 arrivals)
  uint64_t* p_full = bars + 32;     // [unit]  P of a tile is in TMEM (4 arrivals)
  uint64_t* o_full = bars + 34;     // [unit]  one phase per P V
  uint64_t* mma_done = bars + 36;   // [unit] teardown: every MMA issued has completed
  uint64_t* turn_bar = bars + 38;   // [unit][sub-partition] exponential turn of a softmax warp
  constexpr int NBARS = 46;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NBARS + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int npass = p.diff ? 2 : 1;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < NBARS; ++i) mbar_init(&bars[i], (i >= 30 && i < 34) ? 4 : 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    if (p.diff) {
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
  grid_dep_wait();  // the set-up above may run while the previous kernel on the stream retires
  // Register split: the TMA / MMA warpgroup hands registers to the softmax warpgroups, which hold a
  // full 128-column score row. ATT_REGS_LOW * 128 + ATT_REGS_HIGH * 256 stays below the launch's
  // 168 * 384 (static_assert above), so the increase never waits on registers that do not exist.
  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(ATT_REGS_LOW));
    if (warp == 0 || warp == 3) {
      // ---------------------------------------------------------------- TMA producer of unit u
      const int u = warp == 3;
      if (lane == 0) {
        int gk = 0, gv = 0, qc = 0;  // K, V and Q tiles loaded
        bool ok = true;
        for (int item = blockIdx.x; item < num_items && ok; item += gridDim.x) {
          int b, h, tile0;
          decode_item(p, item, pairs_per_head, b, h, tile0);
          const Unit un = make_unit(p, b, tile0 + u);
          if (!un.valid) continue;
          const int nt = un.ntiles, T = npass * nt;
          const int col = h * 64;
          // step n loads K of tile n and V of tile n - 1 (K runs one tile ahead of V)
          for (int n = 0; n <= T && T > 0 && ok; ++n) {
            if (n < T) {
              const int pass = n >= nt;
              const int j = n - pass * nt;
              if (j == 0) {
                const int qs = qc % ATT_QS;
                if (qc >= ATT_QS && !mbar_wait(&q_empty[u * ATT_QS + qs], ((qc / ATT_QS) - 1) & 1, abort_flag, 40)) {
                  ok = false;
                  break;
                }
                mbar_arrive_expect_tx(&q_full[u * ATT_QS + qs], ATT_TILE);
                tma_load_2d(SQ(u, qs), pass ? &tmQ2 : &tmQ, &q_full[u * ATT_QS + qs], col, un.qs + un.i0);
                qc++;
              }
              const int ks = gk % ATT_KS;
              if (gk >= ATT_KS && !mbar_wait(&k_empty[u * ATT_KS + ks], ((gk / ATT_KS) - 1) & 1, abort_flag, 41)) {
                ok = false;
                break;
              }
              mbar_arrive_expect_tx(&k_full[u * ATT_KS + ks], ATT_TILE);
              tma_load_2d(SK(u, ks), pass ? &tmK2 : &tmK, &k_full[u * ATT_KS + ks], col, un.ks + un.j_lo + j * ATT_BN);
              gk++;
            }
            if (n >= 1) {
              const int t = n - 1;
              const int pass = t >= nt;
              const int j = t - pass * nt;
              const int vs = gv % ATT_VS;
              if (gv >= ATT_VS && !mbar_wait(&v_empty[u * ATT_VS + vs], ((gv / ATT_VS) - 1) & 1, abort_flag, 42)) {
                ok = false;
                break;
              }
              mbar_arrive_expect_tx(&v_full[u * ATT_VS + vs], ATT_TILE);
              tma_load_2d(SV(u, vs), pass ? &tmV2 : &tmV, &v_full[u * ATT_VS + vs], col, un.ks + un.j_lo + j * ATT_BN);
              gv++;
            }
          }
        }
        if (*abort_flag) {
          // wait (bounded, ignoring the abort flag) for the last loads this thread issued
          volatile int never = 0;
          for (int c = max(qc - ATT_QS, 0); c < qc; ++c)
            mbar_wait(&q_full[u * ATT_QS + c % ATT_QS], (c / ATT_QS) & 1, &never, 43);
          for (int k = max(gk - ATT_KS, 0); k < gk; ++k)
            mbar_wait(&k_full[u * ATT_KS + k % ATT_KS], (k / ATT_KS) & 1, &never, 43);
          for (int k = max(gv - ATT_VS, 0); k < gv; ++k)
            mbar_wait(&v_full[u * ATT_VS + k % ATT_VS], (k / ATT_VS) & 1, &never, 43);
        }
      }
    } else {
      // ---------------------------------------------------------------- MMA issuer of unit u (whole warp)
      const int u = warp - 1;
      const int fmt = p.f16 ? 0 : 1;
      const uint32_t idesc_s = make_idesc(128, 128, fmt, fmt, 0, 0);
      const uint32_t idesc_o = make_idesc(128, 64, fmt, fmt, 0, 1);
      // Both base words address the start of the tile area; each operand adds the 16-byte-unit offset
      // of its own tile, taken from the same SQ / SK / SV macros that lay the tiles out.
      const uint32_t base = smem_u32(SQ(0, 0));
      const uint64_t dq = sdesc_kmajor_sw128(base);
      const uint64_t dv = sdesc_mnmajor_sw128(base, ATT_TILE);
      const uint32_t k_hi = (uint32_t)(dq >> 32), k_lo = (uint32_t)dq;
      const uint32_t v_hi = (uint32_t)(dv >> 32), v_lo = (uint32_t)dv;
#define OFF16(ptr) ((smem_u32(ptr) - base) >> 4)
      const uint32_t t_s = tmem + 256 * u, t_p = t_s + 128, t_o = t_s + 192;
      int gt = 0, qc = 0;  // tiles and Q tiles consumed
      bool ok = true;
      for (int item = blockIdx.x; item < num_items && ok; item += gridDim.x) {
        int b, h, tile0;
        decode_item(p, item, pairs_per_head, b, h, tile0);
        const Unit un = make_unit(p, b, tile0 + u);
        if (!un.valid) continue;
        const int nt = un.ntiles, T = npass * nt;
        if (T == 0) continue;
        // S of tile 0: the S columns must have been released by the last tile of the previous item
        ok = (gt == 0 || warp_wait(&s_empty[u], (gt - 1) & 1, abort_flag, 44)) &&
             warp_wait(&q_full[u * ATT_QS + qc % ATT_QS], (qc / ATT_QS) & 1, abort_flag, 44) &&
             warp_wait(&k_full[u * ATT_KS + gt % ATT_KS], (gt / ATT_KS) & 1, abort_flag, 45);
        if (!ok) break;
        tc_fence_after();
        {
          const uint32_t qlo = k_lo + OFF16(SQ(u, qc % ATT_QS));
          const uint32_t klo = k_lo + OFF16(SK(u, gt % ATT_KS));
#pragma unroll
          for (int k = 0; k < 4; ++k) mma_ss_lo(t_s, qlo + 2 * k, klo + 2 * k, k_hi, idesc_s, k != 0);
          commit_elect(&s_full[u]);
          commit_elect(&k_empty[u * ATT_KS + gt % ATT_KS]);
          if (nt == 1) commit_elect(&q_empty[u * ATT_QS + qc % ATT_QS]);  // last MMA that reads this Q slot
        }
        for (int t = 0; t < T && ok; ++t) {
          const int g = gt + t;
          if (t + 1 < T) {
            // S of tile t + 1 as soon as the softmax holds tile t in registers
            const int pass1 = (t + 1) >= nt;
            const int j1 = t + 1 - pass1 * nt;
            const int c = qc + pass1;
            ok = warp_wait(&s_empty[u], g & 1, abort_flag, 46) &&
                 (j1 != 0 || warp_wait(&q_full[u * ATT_QS + c % ATT_QS], (c / ATT_QS) & 1, abort_flag, 46)) &&
                 warp_wait(&k_full[u * ATT_KS + (g + 1) % ATT_KS], ((g + 1) / ATT_KS) & 1, abort_flag, 47);
            if (!ok) break;
            tc_fence_after();
            const uint32_t qlo = k_lo + OFF16(SQ(u, c % ATT_QS));
            const uint32_t klo = k_lo + OFF16(SK(u, (g + 1) % ATT_KS));
#pragma unroll
            for (int k = 0; k < 4; ++k) mma_ss_lo(t_s, qlo + 2 * k, klo + 2 * k, k_hi, idesc_s, k != 0);
            commit_elect(&s_full[u]);
            commit_elect(&k_empty[u * ATT_KS + (g + 1) % ATT_KS]);
            if (j1 == nt - 1) commit_elect(&q_empty[u * ATT_QS + c % ATT_QS]);
          }
          // P V of tile t once its P is written
          const int pass = t >= nt;
          const int j = t - pass * nt;
          ok = warp_wait(&p_full[u], g & 1, abort_flag, 48) &&
               warp_wait(&v_full[u * ATT_VS + g % ATT_VS], (g / ATT_VS) & 1, abort_flag, 48);
          if (!ok) break;
          tc_fence_after();
          const uint32_t vlo = v_lo + OFF16(SV(u, g % ATT_VS));
#pragma unroll
          for (int k = 0; k < 8; ++k)
            mma_ts_lo(t_o, t_p + 8 * k, vlo + k * (2048 >> 4), v_hi, idesc_o, (j > 0 || k > 0) ? 1u : 0u);
          commit_elect(&o_full[u]);
          commit_elect(&v_empty[u * ATT_VS + g % ATT_VS]);
        }
        gt += T;
        qc += npass;
      }
#undef OFF16
      // TMEM is released after the final __syncthreads: make sure no MMA of this warp is still running.
      commit_elect(&mma_done[u]);
      volatile int never = 0;
      warp_wait(&mma_done[u], 0, &never, 39);
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(ATT_REGS_HIGH));
    // ------------------------------------------------------------------ softmax warpgroups
    const int u = (warp - 4) >> 2;
    const int wq = warp & 3;  // TMEM lane quarter = SM sub-partition of this warp
    const int r = wq * 32 + lane;
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    const uint32_t t_s = tmem + lane_off + 256 * u;
    const uint32_t t_p = t_s + 128;
    const uint32_t t_o = t_s + 192;
    const float NEG_INF = -INFINITY;
    // Exponential turns: warp wq of unit 0 and warp wq of unit 1 share one sub-partition and its
    // MUFU; they take turns on the exp2 phase, so one warp's loads, maxima and waits run while
    // the other's exponentials keep the MUFU busy. my_turn / next_turn of this warp.
    uint64_t* my_turn = &turn_bar[u * 4 + wq];
    uint64_t* next_turn = &turn_bar[(1 - u) * 4 + wq];
    int turns = 0;
    bool bad_turn = false;
    auto take_turn = [&]() {
      if (u == 1 || turns > 0) {
        const int phase = u == 1 ? turns : turns - 1;
        if (!mbar_wait(my_turn, phase & 1, abort_flag, 53)) bad_turn = true;
      }
    };
    auto pass_turn = [&]() {
      __syncwarp();
      if (lane == 0) mbar_arrive(next_turn);
      turns++;
    };
    int gt = 0;
    float amax = 0.f;
    for (int item = blockIdx.x; item < num_items; item += gridDim.x) {
      int b, h, tile0;
      decode_item(p, item, pairs_per_head, b, h, tile0);
      const Unit un = make_unit(p, b, tile0 + u);
      const Unit uo = make_unit(p, b, tile0 + 1 - u);
      if (!un.valid && !uo.valid) continue;
      const int nt = un.valid ? un.ntiles : 0;
      const int T = npass * nt, To = npass * (uo.valid ? uo.ntiles : 0);
      const int col = h * 64;
      const int i = un.i0 + r;  // query row within its sequence
      const bool row_ok = un.valid && i < un.lq;
      uint16_t* dst = reinterpret_cast<uint16_t*>(p.out) + (long long)(un.qs + i) * p.ldo + col;
      const int lo_j = p.wl < 0 ? 0 : max(0, i + un.dlt - p.wl);
      const int hi_j = p.wr < 0 ? un.lk : min(un.lk, i + un.dlt + p.wr + 1);
      bool bad = false;
      float inv_l = 0.f;
      float m_i = NEG_INF, l_i = 0.f;  // reference maximum (scaled log2 domain) and row sum
      uint32_t park[32];               // differential: stream 1's normalised output, 16-bit pairs
#pragma unroll
      for (int e = 0; e < 32; ++e) park[e] = 0u;

      for (int t = 0; t < max(T, To); ++t) {
        if (t >= T) {
          // the other unit has more tiles in this item: keep the turn sequence in step
          take_turn();
          pass_turn();
          continue;
        }
        const int pass = t >= nt;
        const int j = t - pass * nt;
        if (j == 0) {
          m_i = NEG_INF;
          l_i = 0.f;
        }
        const int g = gt + t;
        if (!mbar_wait(&s_full[u], g & 1, abort_flag, 50)) bad = true;
        tc_fence_after();
        const int j0 = un.j_lo + j * ATT_BN;
        const int clo = lo_j - j0, chi = hi_j - j0;  // visible columns [clo, chi) of this tile
        const bool full = __all_sync(0xffffffffu, clo <= 0 && chi >= ATT_BN);
        // NARROW: bit c is set when 32-column chunk c holds a visible column for some row of this warp;
        // the exponentials of the other chunks are skipped and their P is written as 0, which is what
        // exp2(-inf) gives for their masked scores
        uint32_t need = 0xfu;
        if (NARROW) {
          const int wlo = __reduce_min_sync(0xffffffffu, clo), whi = __reduce_max_sync(0xffffffffu, chi);
          need = 0u;
#pragma unroll
          for (int c = 0; c < 4; ++c)
            if (wlo < 32 * (c + 1) && whi > 32 * c) need |= 1u << c;
        }
        uint32_t sa[32], sb[32], sc[32], sd[32];
        tmem_ld32_async(t_s, sa);
        tmem_ld32_async(t_s + 32, sb);
        tmem_ld32_async(t_s + 64, sc);
        tmem_ld32_async(t_s + 96, sd);
        tmem_wait_ld();
        // the S columns are free for the next tile's Q K^T
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_empty[u]);
        if (!full) {
          mask_chunk(sa, clo, chi);
          mask_chunk(sb, clo - 32, chi - 32);
          mask_chunk(sc, clo - 64, chi - 64);
          mask_chunk(sd, clo - 96, chi - 96);
        }
        float mxs[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) mxs[e] = NEG_INF;
        max_chunk(sa, mxs);
        max_chunk(sb, mxs);
        max_chunk(sc, mxs);
        max_chunk(sd, mxs);
        const float mx = fmaxf(fmax3(fmax3(mxs[0], mxs[1], mxs[2]), mxs[3], mxs[4]),
                               fmax3(mxs[5], mxs[6], mxs[7]));
        const float m_tile = mx * p.scale_log2;  // -inf when no visible key in this tile
        const bool move = m_tile > m_i + ATT_RESCALE_LOG2;
        const float alpha = move ? fast_exp2(m_i - m_tile) : 1.f;  // 0 while m_i = -inf (O row still 0)
        l_i *= alpha;
        // P and O of the previous tile: P V must be done before P is overwritten or O is touched
        if (g > 0 && !mbar_wait(&o_full[u], (g - 1) & 1, abort_flag, 51)) bad = true;
        tc_fence_after();
        // warp-uniform: some row of this warp moves a finite reference maximum
        const bool rescale = __any_sync(0xffffffffu, move && m_i != NEG_INF) && j > 0;
        if (move) m_i = m_tile;
        const float m_use = m_i == NEG_INF ? 0.f : m_i;
        const uint64_t scale2 = f2(p.scale_log2, p.scale_log2), negm2 = f2(-m_use, -m_use);
        uint64_t acc[4] = {0, 0, 0, 0};
        take_turn();
        if (!NARROW) {
          uint32_t w[16];
          exp_chunk(sa, scale2, negm2, acc, w, p.f16);
          tmem_st16(t_p, w);
          exp_chunk(sb, scale2, negm2, acc, w, p.f16);
          tmem_st16(t_p + 16, w);
          exp_chunk(sc, scale2, negm2, acc, w, p.f16);
          tmem_st16(t_p + 32, w);
          exp_chunk(sd, scale2, negm2, acc, w, p.f16);
          tmem_st16(t_p + 48, w);
        } else {
          uint32_t w[16];
          auto chunk = [&](const uint32_t(&sx)[32], uint32_t bit, uint32_t col) {
            if (need & bit) {
              exp_chunk(sx, scale2, negm2, acc, w, p.f16);
            } else {
#pragma unroll
              for (int e = 0; e < 16; ++e) w[e] = 0u;
            }
            tmem_st16(t_p + col, w);
          };
          chunk(sa, 1u, 0);
          chunk(sb, 2u, 16);
          chunk(sc, 4u, 32);
          chunk(sd, 8u, 48);
        }
        pass_turn();
        const float2 r01 = f2_split(fadd2(fadd2(acc[0], acc[1]), fadd2(acc[2], acc[3])));
        l_i += r01.x + r01.y;
        // O work once the score registers are dead, before this tile's P V is released
        if (pass == 1 && j == 0) {
          // end of stream 1: normalise it and keep it in registers as 16-bit pairs (the rounding the
          // reference applies to its first attention output) until stream 2 is done
          uint32_t ov[32];
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            tmem_ld32_async(t_o + 32 * c, ov);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e)
              park[16 * c + e] = pack_2(__uint_as_float(ov[2 * e]) * inv_l, __uint_as_float(ov[2 * e + 1]) * inv_l,
                                        p.f16);
          }
        }
        if (rescale) {
          uint32_t ov[32];
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            tmem_ld32_async(t_o + 32 * c, ov);
            tmem_wait_ld();
            uint32_t w[16];
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {
#pragma unroll
              for (int e = 0; e < 16; ++e) w[e] = __float_as_uint(__uint_as_float(ov[16 * h2 + e]) * alpha);
              tmem_st16(t_o + 32 * c + 16 * h2, w);
            }
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[u]);
        if (j == nt - 1) inv_l = l_i > 0.f ? 1.f / l_i : 0.f;
      }
      gt += T;
      if (!un.valid) continue;

      float o[64];
      if (nt > 0) {
        if (!mbar_wait(&o_full[u], (gt - 1) & 1, abort_flag, 52)) bad = true;
        tc_fence_after();
        uint32_t ov[32];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          tmem_ld32_async(t_o + 32 * c, ov);
          tmem_wait_ld();
#pragma unroll
          for (int d = 0; d < 32; ++d) o[32 * c + d] = __uint_as_float(ov[d]) * inv_l;
        }
        tc_fence_before();
        if (p.diff) {
          // differential combine out - out_diff (transformer.py:790-795), stream 1 from registers
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const uint32_t w = park[e];
            const float lo = p.f16 ? __half2float(__ushort_as_half((unsigned short)(w & 0xffffu)))
                                   : __uint_as_float(w << 16);
            const float hi = p.f16 ? __half2float(__ushort_as_half((unsigned short)(w >> 16)))
                                   : __uint_as_float(w & 0xffff0000u);
            o[2 * e] = lo - o[2 * e];
            o[2 * e + 1] = hi - o[2 * e + 1];
          }
        }
      } else {
#pragma unroll
        for (int d = 0; d < 64; ++d) o[d] = 0.f;
      }
      if (row_ok && !bad && !bad_turn && !*abort_flag) {
        uint32_t pk[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) pk[e] = pack_2(o[2 * e], o[2 * e + 1], p.f16);
#pragma unroll
        for (int qd = 0; qd < 8; ++qd)
          reinterpret_cast<uint4*>(dst)[qd] = make_uint4(pk[4 * qd], pk[4 * qd + 1], pk[4 * qd + 2], pk[4 * qd + 3]);
        if (p.amax_out) {
          // max |y| over the stored 16-bit values; for bf16 the halves widen to f32 with integer shifts and
          // masks, which keeps these conversions off the MUFU that the partner warp's exponentials use
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const uint32_t w = pk[e];
            const float lo = p.f16 ? __half2float(__ushort_as_half((unsigned short)(w & 0xffffu))) : __uint_as_float(w << 16);
            const float hi = p.f16 ? __half2float(__ushort_as_half((unsigned short)(w >> 16))) : __uint_as_float(w & 0xffff0000u);
            amax = fmax3(amax, fabsf(lo), fabsf(hi));
          }
        }
      }
    }
    if (p.amax_out) {
#pragma unroll
      for (int s = 16; s > 0; s >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, s));
      if (lane == 0) atomic_max_nonneg(p.amax_out, amax);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, ATT_TMEM_COLS);
#undef SQ
#undef SK
#undef SV
}

}  // namespace sa3

using namespace sa3;

extern "C" int sa3_attention(const void* q, const void* k, const void* v, const void* q2, const void* k2,
                             const void* v2, void* out, const int* cu_seqlens_q, const int* cu_seqlens_k, int batch,
                             int max_seqlen_q, int max_seqlen_k, int total_q, int total_k, int heads, int head_dim,
                             long long ldq, long long ldk, long long ldv, long long ldo, int window_left,
                             int window_right, float softmax_scale, int dtype, float* amax_out, void* stream) {
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
  p.diff = q2 ? 1 : 0;
  p.out = out;
  p.ldo = ldo;
  p.amax_out = amax_out;
  const int qtiles = (max_seqlen_q + ATT_BM - 1) / ATT_BM;
  const int pairs_per_head = (qtiles + 1) / 2;
  const long long num_items = (long long)pairs_per_head * heads * batch;
  if (num_items > (1LL << 30)) return SA3_ERR_UNSUPPORTED;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    return SA3_ERR_LAUNCH;
  const int grid = num_items < sms ? (int)num_items : sms;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // Narrow windows (the SAME-L window 17) skip the exponentials of the chunks of a tile that no row of a
  // softmax warp sees. SA3_ATT_NARROW=0 / 1 in the environment forces the general / narrow kernel (the
  // two give identical outputs).
  static const int narrow_env = [] {
    const char* e = getenv("SA3_ATT_NARROW");
    return e ? atoi(e) : -1;
  }();
  const bool narrow = narrow_env >= 0 ? narrow_env != 0
                                      : (window_left >= 0 && window_right >= 0 && window_left + window_right + 1 <= 96);
  auto kern = narrow ? attention_tc_kernel<true> : attention_tc_kernel<false>;
  if ((rc = ensure_smem(kern, ATT_SMEM))) return rc;
  launch_ex(kern, dim3(grid), dim3(ATT_THREADS), ATT_SMEM, st, 1, mq, mk, mv, mq2, mk2, mv2, p, (int)num_items,
            pairs_per_head);
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
