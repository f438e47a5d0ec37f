// Sliding-window (and full / cross) attention on tcgen05 for sm_100a.
//
// Replaces the windowed flash-attention call of Attention.apply_attn
// (stable_audio_3/models/transformer.py:620-666, window_size=(wl, wr)) and its
// math-equivalent fallbacks (_sliding_window_chunked_halo_sdpa :143-159,
// _sliding_window_additive_mask :118-127), plus the differential combine
// out - out_diff of Attention.forward (:790-795).
//
// Persistent: one CTA per SM walks work items (query tile fastest, so CTAs that
// run together share K/V tiles in L2); barrier phases run on across items.
// Work unit = 128 query rows x one head x one softmax stream. A CTA runs two
// units side by side: the two streams of a differential head (same rows; the
// combine o1/l1 - o2/l2 happens on chip), or two consecutive query tiles of a
// plain head. 384 threads, warp-specialised:
//   warp 0 (lane 0)  TMA: Q per unit (double-buffered across items), then K and
//                    V tiles through a two-stage ring per unit.
//   warp 1 (lane 0)  tcgen05.mma: S_u = Q_u K^T (M=128, N=128, K=64, both from
//                    shared memory) and O_u += P_u V (M=128, N=64, K=128, P from
//                    TMEM, V MN-major from its TMA tile).
//   warps 4..7, 8..11  softmax warpgroup of unit 0 / unit 1; thread r owns query
//                    row r (TMEM lane r). While one warpgroup runs its softmax the
//                    tensor core works on the other unit's S and P V.
// TMEM per unit (256 columns): S [0,128) fp32, P [128,192) as packed 16-bit
// pairs, O [192,256) fp32. O stays in TMEM for the whole key range; the online
// softmax keeps a reference maximum per row and only moves it (rescaling O and
// the row sum) when a tile's maximum exceeds it by more than 2^8, which keeps
// every exp2 argument <= 8 and leaves the result exactly softmax(S) V. The key
// range of a unit is clipped to the window of its queries, so fully masked key
// tiles are never loaded or multiplied; tiles that lie entirely inside every
// row's band skip masking, edge tiles use one range test per element.
// Shared memory: per unit Q 2x16 KB + K 2x16 KB + V 2x16 KB = 96 KB.
#include "common.cuh"
#include "host_util.h"

namespace sa3 {
SA3_DEFINE_ERROR_READER(read_error_attention)

constexpr int ATT_BM = 128;
constexpr int ATT_BN = 128;
constexpr int ATT_TILE = 128 * 128;  // 128 rows x 64 16-bit elements
constexpr int ATT_UNIT_TILES = 6;    // Q0, Q1, K0, K1, V0, V1
constexpr int ATT_THREADS = 384;
constexpr int ATT_SMEM = 2 * ATT_UNIT_TILES * ATT_TILE + 1024 + 1024;  // tiles + barriers, slots, row-sum exchange
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

__global__ void __launch_bounds__(ATT_THREADS, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmQ2,
                        const __grid_constant__ CUtensorMap tmK2, const __grid_constant__ CUtensorMap tmV2,
                        AttnParams p, int num_items, int pairs_per_head) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
#define SQ(u, b) (smem + ((u) * ATT_UNIT_TILES + (b)) * ATT_TILE)
#define SK(u, s) (smem + ((u) * ATT_UNIT_TILES + 2 + (s)) * ATT_TILE)
#define SV(u, s) (smem + ((u) * ATT_UNIT_TILES + 4 + (s)) * ATT_TILE)
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 2 * ATT_UNIT_TILES * ATT_TILE);
  uint64_t* q_full = bars;         // [unit][slot]
  uint64_t* q_empty = bars + 4;    // [unit][slot]
  uint64_t* kv_full = bars + 8;    // [unit][stage]
  uint64_t* kv_empty = bars + 12;  // [unit][stage]
  uint64_t* s_full = bars + 16;    // [unit]
  uint64_t* p_full = bars + 18;    // [unit]  (4 arrivals: one per softmax warp)
  uint64_t* o_full = bars + 20;    // [unit]  one phase per P V
  uint64_t* mma_done = bars + 22;  // teardown: every MMA issued has completed
  constexpr int NBARS = 23;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NBARS + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int npass = p.diff ? 2 : 1;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < NBARS; ++i) mbar_init(&bars[i], (i == 18 || i == 19) ? 4 : 1);
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
  // Register split: the TMA / MMA warpgroup hands registers to the softmax warpgroups, which hold a
  // full 128-column score row. ATT_REGS_LOW * 128 + ATT_REGS_HIGH * 256 stays below the launch's
  // 168 * 384 (static_assert above), so the increase never waits on registers that do not exist.
  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(ATT_REGS_LOW));
    if (warp == 0) {
      // ---------------------------------------------------------------- TMA producer
      if (lane == 0) {
        int gk[2] = {0, 0};  // K/V tiles loaded per unit
        int qc[2] = {0, 0};  // Q tiles loaded per unit
        bool ok = true;
        for (int item = blockIdx.x; item < num_items && ok; item += gridDim.x) {
          int b, h, tile0;
          decode_item(p, item, pairs_per_head, b, h, tile0);
          const Unit U0 = make_unit(p, b, tile0);
          if (!U0.valid) continue;
          const Unit U1 = make_unit(p, b, tile0 + 1);
          const int nt[2] = {U0.ntiles, U1.valid ? U1.ntiles : 0};
          const int T0 = npass * nt[0], T1 = npass * nt[1];
          const int col = h * 64;
          for (int t = 0; t < max(T0, T1) && ok; ++t) {
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              if (t >= (u ? T1 : T0) || !ok) continue;
              const Unit& un = u ? U1 : U0;
              const int pass = t >= nt[u];
              const int j = t - pass * nt[u];
              if (j == 0) {
                const int c = qc[u], qs = c & 1;
                if (c >= 2 && !mbar_wait(&q_empty[u * 2 + qs], ((c >> 1) - 1) & 1, abort_flag, 40)) {
                  ok = false;
                  continue;
                }
                mbar_arrive_expect_tx(&q_full[u * 2 + qs], ATT_TILE);
                tma_load_2d(SQ(u, qs), pass ? &tmQ2 : &tmQ, &q_full[u * 2 + qs], col, un.qs + un.i0);
                qc[u]++;
              }
              const int g = gk[u];
              const int s = g & 1;
              if (g >= 2 && !mbar_wait(&kv_empty[u * 2 + s], ((g >> 1) - 1) & 1, abort_flag, 41)) {
                ok = false;
                continue;
              }
              const int row = un.ks + un.j_lo + j * ATT_BN;
              mbar_arrive_expect_tx(&kv_full[u * 2 + s], 2 * ATT_TILE);
              tma_load_2d(SK(u, s), pass ? &tmK2 : &tmK, &kv_full[u * 2 + s], col, row);
              tma_load_2d(SV(u, s), pass ? &tmV2 : &tmV, &kv_full[u * 2 + s], col, row);
              gk[u]++;
            }
          }
        }
        if (*abort_flag) {
          // wait (bounded, ignoring the abort flag) for the last loads this thread issued
          volatile int never = 0;
          for (int u = 0; u < 2; ++u) {
            for (int c = qc[u] - 2; c < qc[u]; ++c)
              if (c >= 0) mbar_wait(&q_full[u * 2 + (c & 1)], (c >> 1) & 1, &never, 42);
            for (int k = gk[u] - 2; k < gk[u]; ++k)
              if (k >= 0) mbar_wait(&kv_full[u * 2 + (k & 1)], (k >> 1) & 1, &never, 43);
          }
        }
      }
    } else if (warp == 1) {
      // ---------------------------------------------------------------- MMA issuer (whole warp)
      const int fmt = p.f16 ? 0 : 1;
      const uint32_t idesc_s = make_idesc(128, 128, fmt, fmt, 0, 0);
      const uint32_t idesc_o = make_idesc(128, 64, fmt, fmt, 0, 1);
      // Descriptors differ only in their start-address field (low word, in 16-byte units), and every
      // tile of the ring sits at a fixed offset, so each MMA only adds a constant to one 32-bit word.
      // Both base words address the start of the tile area; each operand adds the 16-byte-unit offset
      // of its own tile, taken from the same SQ / SK / SV macros that lay the tiles out.
      const uint32_t base = smem_u32(SQ(0, 0));
      const uint64_t dq = sdesc_kmajor_sw128(base);
      const uint64_t dv = sdesc_mnmajor_sw128(base, ATT_TILE);
      const uint32_t k_hi = (uint32_t)(dq >> 32), k_lo = (uint32_t)dq;
      const uint32_t v_hi = (uint32_t)(dv >> 32), v_lo = (uint32_t)dv;
#define OFF16(ptr) ((smem_u32(ptr) - base) >> 4)
      int gk[2] = {0, 0};
      int qc[2] = {0, 0};
      bool ok = true;
      for (int item = blockIdx.x; item < num_items && ok; item += gridDim.x) {
        int b, h, tile0;
        decode_item(p, item, pairs_per_head, b, h, tile0);
        const Unit U0 = make_unit(p, b, tile0);
        if (!U0.valid) continue;
        const Unit U1 = make_unit(p, b, tile0 + 1);
        const int nt[2] = {U0.ntiles, U1.valid ? U1.ntiles : 0};
        const int T[2] = {npass * nt[0], npass * nt[1]};
        // first S of each unit: Q of pass 0, first K tile
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          if (T[u] == 0 || !ok) continue;
          const int g = gk[u], c = qc[u];
          ok = warp_wait(&q_full[u * 2 + (c & 1)], (c >> 1) & 1, abort_flag, 44) &&
               warp_wait(&kv_full[u * 2 + (g & 1)], (g >> 1) & 1, abort_flag, 45);
          if (!ok) continue;
          tc_fence_after();
          const uint32_t qlo = k_lo + OFF16(SQ(u, c & 1));
          const uint32_t klo = k_lo + OFF16(SK(u, g & 1));
#pragma unroll
          for (int k = 0; k < 4; ++k) mma_ss_lo(tmem + 256 * u, qlo + 2 * k, klo + 2 * k, k_hi, idesc_s, k != 0);
          commit_elect(&s_full[u]);
          if (nt[u] == 1) commit_elect(&q_empty[u * 2 + (c & 1)]);  // last MMA that reads this Q slot
        }
        for (int t = 0; t < max(T[0], T[1]) && ok; ++t) {
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            if (t >= T[u] || !ok) continue;
            const int g = gk[u] + t;
            const int s = g & 1;
            const int pass = t >= nt[u];
            const int j = t - pass * nt[u];
            if (!warp_wait(&p_full[u], g & 1, abort_flag, 46)) {
              ok = false;
              continue;
            }
            tc_fence_after();
            // O_pass (+)= P V: P is the 16-bit copy the softmax wrote over the first 64 columns of S
            const uint32_t vlo = v_lo + OFF16(SV(u, s));
#pragma unroll
            for (int k = 0; k < 8; ++k)
              mma_ts_lo(tmem + 256 * u + 128 + 64 * pass, tmem + 256 * u + 8 * k, vlo + k * (2048 >> 4), v_hi, idesc_o,
                        (j > 0 || k > 0) ? 1u : 0u);
            commit_elect(&o_full[u]);
            commit_elect(&kv_empty[u * 2 + s]);
            if (t + 1 < T[u]) {
              // S of the next tile overwrites the P just read: tcgen05 MMAs execute in issue order
              const int pass1 = (t + 1) >= nt[u];
              const int j1 = t + 1 - pass1 * nt[u];
              const int c = qc[u] + pass1;
              const int s1 = (g + 1) & 1;
              if ((j1 == 0 && !warp_wait(&q_full[u * 2 + (c & 1)], (c >> 1) & 1, abort_flag, 47)) ||
                  !warp_wait(&kv_full[u * 2 + s1], ((g + 1) >> 1) & 1, abort_flag, 48)) {
                ok = false;
                continue;
              }
              tc_fence_after();
              const uint32_t qlo = k_lo + OFF16(SQ(u, c & 1));
              const uint32_t klo = k_lo + OFF16(SK(u, s1));
#pragma unroll
              for (int k = 0; k < 4; ++k)
                mma_ss_lo(tmem + 256 * u, qlo + 2 * k, klo + 2 * k, k_hi, idesc_s, k != 0);
              commit_elect(&s_full[u]);
              if (j1 == nt[u] - 1) commit_elect(&q_empty[u * 2 + (c & 1)]);
            }
          }
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          if (T[u] == 0) continue;
          gk[u] += T[u];
          qc[u] += npass;
        }
      }
      // TMEM is released after the final __syncthreads: make sure no MMA is still running then.
      commit_elect(mma_done);
      volatile int never = 0;
      warp_wait(mma_done, 0, &never, 39);
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(ATT_REGS_HIGH));
    // ------------------------------------------------------------------ softmax warpgroups
    const int u = (warp - 4) >> 2;
    const int wq = warp & 3;  // TMEM lane quarter
    const int r = wq * 32 + lane;
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    const uint32_t t_s = tmem + lane_off + 256 * u;  // S, then P over its first 64 columns
    const float NEG_INF = -INFINITY;
    int gk = 0;
    float amax = 0.f;
    for (int item = blockIdx.x; item < num_items; item += gridDim.x) {
      int b, h, tile0;
      decode_item(p, item, pairs_per_head, b, h, tile0);
      const Unit un = make_unit(p, b, tile0 + u);
      if (!un.valid) continue;
      const int col = h * 64;
      const int i = un.i0 + r;  // query row within its sequence
      const int lo_j = p.wl < 0 ? 0 : max(0, i + un.dlt - p.wl);
      const int hi_j = p.wr < 0 ? un.lk : min(un.lk, i + un.dlt + p.wr + 1);
      float inv_l[2] = {0.f, 0.f};
      bool bad = false;

      for (int pass = 0; pass < npass; ++pass) {
        const uint32_t t_o = t_s + 128 + 64 * pass;
        float m_i = NEG_INF, l_i = 0.f;  // reference maximum (scaled log2 domain) and row sum
        for (int j = 0; j < un.ntiles; ++j) {
          const int g = gk + pass * un.ntiles + j;
          if (!mbar_wait(&s_full[u], g & 1, abort_flag, 50)) bad = true;
          tc_fence_after();
          const int j0 = un.j_lo + j * ATT_BN;
          const int clo = lo_j - j0, chi = hi_j - j0;  // visible columns [clo, chi) of this tile
          const bool full = __all_sync(0xffffffffu, clo <= 0 && chi >= ATT_BN);
          uint32_t sa[32], sb[32], sc[32], sd[32];
          tmem_ld32_async(t_s, sa);
          tmem_ld32_async(t_s + 32, sb);
          tmem_ld32_async(t_s + 64, sc);
          tmem_ld32_async(t_s + 96, sd);
          tmem_wait_ld();
          if (!full) {
            mask_chunk(sa, clo, chi);
            mask_chunk(sb, clo - 32, chi - 32);
            mask_chunk(sc, clo - 64, chi - 64);
            mask_chunk(sd, clo - 96, chi - 96);
          }
          float mxs[8];
#pragma unroll
          for (int t = 0; t < 8; ++t) mxs[t] = NEG_INF;
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
          // warp-uniform: some row of this warp moves a finite reference maximum
          const bool rescale = __any_sync(0xffffffffu, move && m_i != NEG_INF) && j > 0;
          if (rescale) {
            // rescale O once the previous P V has landed in it
            if (!mbar_wait(&o_full[u], (g - 1) & 1, abort_flag, 51)) bad = true;
            tc_fence_after();
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
          if (move) m_i = m_tile;
          const float m_use = m_i == NEG_INF ? 0.f : m_i;
          const uint64_t scale2 = f2(p.scale_log2, p.scale_log2), negm2 = f2(-m_use, -m_use);
          uint64_t acc[4] = {0, 0, 0, 0};
          {
            uint32_t w[16];
            exp_chunk(sa, scale2, negm2, acc, w, p.f16);
            tmem_st16(t_s, w);
            exp_chunk(sb, scale2, negm2, acc, w, p.f16);
            tmem_st16(t_s + 16, w);
            exp_chunk(sc, scale2, negm2, acc, w, p.f16);
            tmem_st16(t_s + 32, w);
            exp_chunk(sd, scale2, negm2, acc, w, p.f16);
            tmem_st16(t_s + 48, w);
          }
          const float2 r01 = f2_split(fadd2(fadd2(acc[0], acc[1]), fadd2(acc[2], acc[3])));
          l_i += r01.x + r01.y;
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&p_full[u]);
        }
        inv_l[pass] = l_i > 0.f ? 1.f / l_i : 0.f;
      }
      gk += npass * un.ntiles;

      float o[64];
      if (un.ntiles > 0) {
        if (!mbar_wait(&o_full[u], (gk - 1) & 1, abort_flag, 49)) bad = true;
        tc_fence_after();
        uint32_t ov[32];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          tmem_ld32_async(t_s + 128 + 32 * c, ov);
          tmem_wait_ld();
#pragma unroll
          for (int d = 0; d < 32; ++d) o[32 * c + d] = __uint_as_float(ov[d]) * inv_l[0];
        }
        if (p.diff) {
          // differential combine o1 / l1 - o2 / l2 (transformer.py:790-795)
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            tmem_ld32_async(t_s + 192 + 32 * c, ov);
            tmem_wait_ld();
#pragma unroll
            for (int d = 0; d < 32; ++d) o[32 * c + d] = fmaf(-__uint_as_float(ov[d]), inv_l[1], o[32 * c + d]);
          }
        }
        tc_fence_before();
      } else {
#pragma unroll
        for (int d = 0; d < 64; ++d) o[d] = 0.f;
      }
      if (i < un.lq && !bad && !*abort_flag) {
        uint16_t* dst = reinterpret_cast<uint16_t*>(p.out) + (long long)(un.qs + i) * p.ldo + col;
#pragma unroll
        for (int qd = 0; qd < 8; ++qd) {
          uint4 w;
          w.x = pack_2(o[qd * 8 + 0], o[qd * 8 + 1], p.f16);
          w.y = pack_2(o[qd * 8 + 2], o[qd * 8 + 3], p.f16);
          w.z = pack_2(o[qd * 8 + 4], o[qd * 8 + 5], p.f16);
          w.w = pack_2(o[qd * 8 + 6], o[qd * 8 + 7], p.f16);
          reinterpret_cast<uint4*>(dst)[qd] = w;
        }
        if (p.amax_out) {
#pragma unroll
          for (int d = 0; d < 64; ++d)
            amax = fmaxf(amax, fabsf(p.f16 ? __half2float(__float2half(o[d]))
                                           : __bfloat162float(__float2bfloat16(o[d]))));
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
#undef OFF16
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
  if ((rc = ensure_smem(attention_tc_kernel, ATT_SMEM))) return rc;
  attention_tc_kernel<<<grid, ATT_THREADS, ATT_SMEM, st>>>(mq, mk, mv, mq2, mk2, mv2, p, (int)num_items,
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
