// tcgen05 GEMM for the DiT linears: C = epilogue(A . B^T * a_scale * b_scale[n] + bias[n]).
//
// Replaces the nn.Linear projections of stable_audio_3/models/transformer.py
// (Attention.to_qkv/to_q/to_kv/to_out :547-560, GLU.proj :432, FeedForward
// linear_out :485, TransformerBlock.to_local_embed :944-957) with FP8 e4m3 or
// bf16 operands, and fuses the adaLN gate + residual of TransformerBlock.forward
// (:1027-1029, :1047-1049), the SwiGLU of GLU.forward (:443-444) and the
// local-conditioning left-pad add (_left_pad_to_match :77-88) into the epilogue.
//
// Structure (one 128 x 256 output tile per CTA, 128 threads):
//   warp 0 / lane 0 : TMA producer, STAGES-deep ring of (A 128x128B, B 256x128B)
//                     tiles with the 128-byte swizzle, one mbarrier per stage.
//   warp 1 / lane 0 : tcgen05.mma issuer (M=128, N=256, K=16 bf16 or K=32 fp8
//                     per instruction), accumulator in 256 TMEM columns.
//   all 4 warps     : epilogue; warp w owns TMEM lanes / tile rows 32w..32w+31.
#include "common.cuh"
#include "host_util.h"

namespace sa3 {
SA3_DEFINE_ERROR_READER(read_error_gemm)
int read_error_glue(int* out);
int read_error_attention(int* out);
int read_error_peer(int* out);

constexpr int GEMM_BM = 128;
constexpr int GEMM_BN = 256;
constexpr int GEMM_STAGES = 4;
constexpr int GEMM_A_BYTES = GEMM_BM * 128;
constexpr int GEMM_B_BYTES = GEMM_BN * 128;
constexpr int GEMM_STAGE_BYTES = GEMM_A_BYTES + GEMM_B_BYTES;
constexpr int GEMM_SMEM = GEMM_STAGES * GEMM_STAGE_BYTES + 1024 /*align slack*/ + 256 /*barriers*/;
constexpr int GEMM_TMEM_COLS = 256;

struct GemmParams {
  int M, N, K;
  long long ldc;
  void* C;
  const float* a_scale;
  const float* b_scale;
  sa3_epilogue epi;
  int tma_store;  // 1: bf16 output through shared memory and TMA stores (no output-row remap);
                  // 2: fp32 residual in and result out through TMA; 3: in-place fp32 residual by TMA reduce-add
};

// bf16 output chunks of 32 rows x 32 columns go out through a per-warp double buffer in shared
// memory and one TMA store each. The buffers use the 64-byte swizzle of the output tensor map, so
// the row writes below are free of bank conflicts; a buffer is reused only after the TMA store
// that last read it has finished reading (bulk-group wait).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* m, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
// Element-wise add of a shared-memory box into global memory, performed at L2 (fp32 add, rounded to
// nearest even); the box is read from shared memory asynchronously like a TMA store.
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* m, const void* src, int x, int y) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_all_but_one() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

struct StoreStage {
  const CUtensorMap* tm;   // output map: box 32 x 32 bf16, or 16 x 32 fp32 (residual kinds); 64-byte swizzle
  const CUtensorMap* tmr;  // residual map (fp32 residual kinds): box 16 x 32 fp32, 64-byte swizzle
  uint8_t* buf;            // this warp's 2 x 2 KB, 512-byte aligned
  uint64_t* rbar;          // this warp's 2 residual-load barriers
  volatile int* abort;
  int next;                // bf16: buffer to fill next
  int uses;                // residual: chunks loaded so far (barrier phase)
  int pending;             // residual: loads issued and not yet consumed
  int red;                 // in-place residual kinds: the result is added into C by TMA reduce-add
  int f16;                 // reduce-add into an fp16 C: one 32 x 32 box per chunk, buffers alternate by `next`
};

// This thread's row of the chunk (v, columns col..col+31 of output row row0 + lane) -> bf16 -> TMA.
__device__ __forceinline__ void stage_store32(StoreStage& st, int col, int row0, int M, const float (&v)[32],
                                              float& amax, bool want_amax) {
  const int lane = threadIdx.x & 31;
  uint8_t* b = st.buf + st.next * 2048;
  if (lane == 0) bulk_wait_read_all_but_one();  // the store issued two chunks ago has read this buffer
  __syncwarp();
  uint32_t w[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) w[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
  if (want_amax && row0 + lane < M) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
      amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
    }
  }
#pragma unroll
  for (int c = 0; c < 4; ++c)
    *reinterpret_cast<uint4*>(b + lane * 64 + ((c ^ ((lane >> 1) & 3)) * 16)) =
        make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0 && row0 < M) {  // rows past M are clipped by the tensor map; a box wholly past M is skipped
    tma_store_2d(st.tm, b, col, row0);
    bulk_commit_group();
  }
  st.next ^= 1;
}

__device__ __forceinline__ int out_row_of(const sa3_epilogue& e, int m) {
  if (e.out_row_map) return __ldg(e.out_row_map + m);
  return e.seg_in > 0 ? (m / e.seg_in) * e.seg_out + e.seg_offset + (m % e.seg_in) : m;
}

__device__ __forceinline__ void load_bf16x32(const __nv_bfloat16* p, float (&v)[32]) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 u = q[i];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __bfloat1622float2(h[j]);
      v[i * 8 + 2 * j] = f.x;
      v[i * 8 + 2 * j + 1] = f.y;
    }
  }
}

__device__ __forceinline__ void load_f16x32(const __half* p, float (&v)[32]) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 u = q[i];
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __half22float2(h[j]);
      v[i * 8 + 2 * j] = f.x;
      v[i * 8 + 2 * j + 1] = f.y;
    }
  }
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void load_f32x32(const float* p, float (&v)[32]) {
  const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float4 u = q[i];
    v[4 * i] = u.x;
    v[4 * i + 1] = u.y;
    v[4 * i + 2] = u.z;
    v[4 * i + 3] = u.w;
  }
}

__device__ __forceinline__ void store_f32x32(float* p, const float (&v)[32]) {
  float4* q = reinterpret_cast<float4*>(p);
#pragma unroll
  for (int i = 0; i < 8; ++i) q[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* p, const float (&v)[32]) {
  uint4* q = reinterpret_cast<uint4*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 u;
    u.x = pack_bf16x2(v[i * 8 + 0], v[i * 8 + 1]);
    u.y = pack_bf16x2(v[i * 8 + 2], v[i * 8 + 3]);
    u.z = pack_bf16x2(v[i * 8 + 4], v[i * 8 + 5]);
    u.w = pack_bf16x2(v[i * 8 + 6], v[i * 8 + 7]);
    q[i] = u;
  }
}

// Scale + bias of one 32-column chunk starting at weight row n (bounds-checked).
__device__ __forceinline__ void apply_scale_bias(float (&v)[32], int n, int N, float sa, const float* b_scale,
                                                 const float* bias) {
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int c = n + i;
    float s = sa;
    float b = 0.f;
    if (c < N) {
      if (b_scale) s *= __ldg(b_scale + c);
      if (bias) b = __ldg(bias + c);
    }
    v[i] = v[i] * s + b;
  }
}

template <bool FP8>
__global__ void __launch_bounds__(128, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + GEMM_STAGES * GEMM_STAGE_BYTES);
  uint64_t* empty = full + GEMM_STAGES;
  uint64_t* accf = empty + GEMM_STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accf + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * GEMM_BN;
  const int m0 = blockIdx.y * GEMM_BM;
  constexpr int BK = FP8 ? 128 : 64;  // elements per 128-byte row
  const int nkb = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < GEMM_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accf, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, GEMM_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dep_wait();  // the set-up above may run while the previous kernel on the stream retires

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer
    int issued = 0;
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % GEMM_STAGES;
      if (kb >= GEMM_STAGES) {
        if (!mbar_wait(&empty[s], ((kb / GEMM_STAGES) - 1) & 1, abort_flag, 1)) break;
      }
      uint8_t* st = smem + s * GEMM_STAGE_BYTES;
      mbar_arrive_expect_tx(&full[s], GEMM_STAGE_BYTES);
      tma_load_2d(st, &tmA, &full[s], kb * BK, m0);
      tma_load_2d(st + GEMM_A_BYTES, &tmB, &full[s], kb * BK, n0);
      issued = kb + 1;
    }
    if (*abort_flag) {
      // Drain the loads still in flight before the CTA may exit.
      for (int kb = (issued > GEMM_STAGES ? issued - GEMM_STAGES : 0); kb < issued; ++kb) {
        volatile int never = 0;
        mbar_wait(&full[kb % GEMM_STAGES], (kb / GEMM_STAGES) & 1, &never, 4);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer
    const uint32_t idesc = make_idesc(GEMM_BM, GEMM_BN, FP8 ? 0 : 1, FP8 ? 0 : 1, 0, 0);
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % GEMM_STAGES;
      if (!mbar_wait(&full[s], (kb / GEMM_STAGES) & 1, abort_flag, 2)) break;
      tc_fence_after();
      const uint32_t a_addr = smem_u32(smem + s * GEMM_STAGE_BYTES);
      const uint64_t ad = sdesc_kmajor_sw128(a_addr);
      const uint64_t bd = sdesc_kmajor_sw128(a_addr + GEMM_A_BYTES);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        // Each K step consumes 32 bytes of the 128-byte swizzled row: +2 in the
        // (address >> 4) field of both descriptors.
        if (FP8)
          mma_f8_ss(tmem, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
        else
          mma_f16_ss(tmem, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
      }
      tc_commit(&empty[s]);
    }
    tc_commit(accf);
  }
  __syncwarp();

  // ---------------- epilogue
  const bool ok = mbar_wait(accf, 0, abort_flag, 3);
  tc_fence_after();
  if (ok && !*abort_flag) {
    const sa3_epilogue& e = p.epi;
    const int m = m0 + warp * 32 + lane;
    const bool row_ok = m < p.M;
    const float sa = p.a_scale ? __ldg(p.a_scale) : 1.f;
    const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
    __nv_bfloat16* C = reinterpret_cast<__nv_bfloat16*>(p.C);
    const int orow = out_row_of(e, m);
    float amax = 0.f;
    int batch = 0;
    if (e.kind == SA3_EPI_GATED_RESIDUAL && row_ok)
      batch = e.row_batch ? __ldg(e.row_batch + m) : (e.rows_per_batch > 0 ? m / e.rows_per_batch : 0);

    if (e.kind == SA3_EPI_SWIGLU) {
      // Tile columns [0,128) hold x rows, [128,256) the matching gate rows.
      const int Nout = p.N / 2;
      const int nout0 = n0 / 2;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float x[32], g[32];
        tmem_ld32(trow + c * 32, x);
        tmem_ld32(trow + 128 + c * 32, g);
        apply_scale_bias(x, n0 + c * 32, p.N, sa, p.b_scale, e.bias);
        apply_scale_bias(g, n0 + 128 + c * 32, p.N, sa, p.b_scale, e.bias);
        float y[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) y[i] = x[i] * siluf_(g[i]);
        const int nc = nout0 + c * 32;
        if (row_ok && nc < Nout) {
          __nv_bfloat16* dst = C + (long long)orow * p.ldc + nc;
          if (nc + 32 <= Nout && (p.ldc & 7) == 0 && (reinterpret_cast<uintptr_t>(p.C) & 15) == 0) {
            store_bf16x32(dst, y);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (nc + i < Nout) dst[i] = __float2bfloat16(y[i]);
          }
#pragma unroll
          for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(__bfloat162float(__float2bfloat16(y[i]))));
        }
      }
    } else {
#pragma unroll 1
      for (int c = 0; c < GEMM_BN / 32; ++c) {
        const int nc = n0 + c * 32;
        if (nc >= p.N) break;  // uniform across the CTA
        float v[32];
        tmem_ld32(trow + c * 32, v);
        apply_scale_bias(v, nc, p.N, sa, p.b_scale, e.bias);
        const bool full_chunk = (nc + 32 <= p.N) && ((p.ldc & 7) == 0) && ((e.ld_residual & 7) == 0) &&
                                ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0) &&
                                ((reinterpret_cast<uintptr_t>(e.residual) & 15) == 0);
        if (e.kind == SA3_EPI_SILU) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = siluf_(v[i]);
        } else if (e.kind == SA3_EPI_GATED_RESIDUAL || e.kind == SA3_EPI_RESIDUAL) {
          if (row_ok) {
            float r[32];
            if (e.c_f32) {
              const float* res = reinterpret_cast<const float*>(e.residual) + (long long)orow * e.ld_residual + nc;
              if (full_chunk) {
                load_f32x32(res, r);
              } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) r[i] = (nc + i < p.N) ? res[i] : 0.f;
              }
            } else {
              const __nv_bfloat16* res =
                  reinterpret_cast<const __nv_bfloat16*>(e.residual) + (long long)orow * e.ld_residual + nc;
              if (full_chunk) {
                load_bf16x32(res, r);
              } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) r[i] = (nc + i < p.N) ? __bfloat162float(res[i]) : 0.f;
              }
            }
            if (e.kind == SA3_EPI_GATED_RESIDUAL) {
              const float* gt = e.gate + (long long)batch * e.ld_gate + nc;
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                const float gv = (nc + i < p.N) ? __ldg(gt + i) : 0.f;
                v[i] = r[i] + v[i] * sigmoidf_(1.f - gv);
              }
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = r[i] + v[i];
            }
          }
        }
        if (row_ok) {
          if (e.c_f32) {
            float* dst = reinterpret_cast<float*>(p.C) + (long long)orow * p.ldc + nc;
            if (full_chunk) {
              store_f32x32(dst, v);
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (nc + i < p.N) dst[i] = v[i];
            }
          } else {
            __nv_bfloat16* dst = C + (long long)orow * p.ldc + nc;
            if (full_chunk) {
              store_bf16x32(dst, v);
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (nc + i < p.N) dst[i] = __float2bfloat16(v[i]);
            }
          }
          if (e.amax_out) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (nc + i < p.N)
                amax = fmaxf(amax, fabsf(e.c_f32 ? v[i] : __bfloat162float(__float2bfloat16(v[i]))));
          }
        }
      }
    }
    if (e.amax_out) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      if (lane == 0) atomic_max_nonneg(e.amax_out, amax);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, GEMM_TMEM_COLS);
}


// ---------------------------------------------------------------------------------------------
// Persistent variant: one CTA per SM walks output tiles (n fastest) with a static stride.
//   warp 0 / lane 0 : TMA producer over a STAGES-deep ring that runs on across tiles.
//   warp 1 / lane 0 : MMA issuer; the accumulator alternates between two 256-column TMEM
//                     buffers, so tile i+1's main loop overlaps tile i's epilogue.
//   warps 2..9      : epilogue; warp w reads TMEM lane quarter w % 4 and column half (w - 2) / 4,
//                     vectorised loads of per-column scale / bias / gate, 16-byte stores.
// Requirements (checked on the host): N % 32 == 0 (N % 256 for SwiGLU), 16-byte aligned C,
// residual, b_scale, bias and gate rows.
constexpr int PG_THREADS = 320;
constexpr int PG_EPI_WARPS = 8;
constexpr int PG_TMEM_COLS = 512;
// Epilogue region, shared by the persistent kernels: the per-warp transpose scratch (8 warps x 32 x 33 floats)
// and, on the same bytes, the per-warp 2 x 2 KB TMA-store staging buffers (512-byte aligned); the 2 residual-load
// mbarriers of each warp follow the whole region, so no data store ever lands on a live mbarrier object.
constexpr int PG_SCRATCH_BYTES = PG_EPI_WARPS * 32 * 33 * 4;
constexpr int PG_STAGING_BYTES = PG_EPI_WARPS * 4096;
constexpr int PG_RBAR_BYTES = 2 * PG_EPI_WARPS * 8;
static_assert(PG_STAGING_BYTES + 511 <= PG_SCRATCH_BYTES, "TMA-store staging must fit inside the epilogue region");
// byte offset of the residual-load barriers from the start of the epilogue region
__host__ __device__ constexpr int pg_rbar_offset() { return PG_SCRATCH_BYTES; }
// ring | barriers (256 B) | epilogue region | residual barriers; + 1 KB alignment slack
constexpr int PG_SCRATCH_OFFSET = GEMM_STAGES * GEMM_STAGE_BYTES + 256;
constexpr int PG_SMEM = PG_SCRATCH_OFFSET + PG_SCRATCH_BYTES + PG_RBAR_BYTES + 1024;
static_assert(PG_SCRATCH_OFFSET % 8 == 0 && PG_SCRATCH_BYTES % 8 == 0, "mbarriers need 8-byte alignment");
static_assert(PG_SMEM <= 232448, "persistent GEMM exceeds the 227 KB shared-memory limit");

// sigmoid(x) = (1 + tanh(x / 2)) / 2: one MUFU operation (tanh.approx, relative error ~2^-11) instead of an
// exponential and a reciprocal; the epilogues that use it write bf16 or feed an fp32 residual update.
__device__ __forceinline__ float fast_sigmoid(float x) {
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(0.5f * x));
  return fmaf(0.5f, t, 0.5f);
}

__device__ __forceinline__ void ldg_f32x32(const float* p, float (&v)[32]) {
  const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 u = __ldg(q + i);
    v[4 * i] = u.x;
    v[4 * i + 1] = u.y;
    v[4 * i + 2] = u.z;
    v[4 * i + 3] = u.w;
  }
}

// acc * sa * b_scale[n] + bias[n] for 32 columns starting at n (vectorised, no bounds checks).
__device__ __forceinline__ void scale_bias32(float (&v)[32], int n, float sa, const float* b_scale,
                                             const float* bias) {
  if (b_scale) {
    float s[32];
    ldg_f32x32(b_scale + n, s);
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] *= sa * s[i];
  } else if (sa != 1.f) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] *= sa;
  }
  if (bias) {
    float b[32];
    ldg_f32x32(bias + n, b);
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] += b[i];
  }
}

template <int KIND>
__device__ __forceinline__ void pg_store_chunk(const GemmParams& p, int m, int orow, int batch, int nc, float (&v)[32],
                                               float& amax) {
  const sa3_epilogue& e = p.epi;
  if (KIND == SA3_EPI_SILU) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = v[i] * fast_sigmoid(v[i]);
  }
  if (m >= p.M) return;
  if (KIND == SA3_EPI_GATED_RESIDUAL || KIND == SA3_EPI_RESIDUAL) {
    float r[32];
    if (e.c_f32)
      load_f32x32(reinterpret_cast<const float*>(e.residual) + (long long)orow * e.ld_residual + nc, r);
    else if (e.c_f16)
      load_f16x32(reinterpret_cast<const __half*>(e.residual) + (long long)orow * e.ld_residual + nc, r);
    else
      load_bf16x32(reinterpret_cast<const __nv_bfloat16*>(e.residual) + (long long)orow * e.ld_residual + nc, r);
    if (KIND == SA3_EPI_GATED_RESIDUAL) {
      float g[32];
      ldg_f32x32(e.gate + (long long)batch * e.ld_gate + nc, g);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = r[i] + v[i] * fast_sigmoid(1.f - g[i]);
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] += r[i];
    }
  }
  if (e.c_f32) {
    store_f32x32(reinterpret_cast<float*>(p.C) + (long long)orow * p.ldc + nc, v);
    if (e.amax_out) {
#pragma unroll
      for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    }
  } else if (e.c_f16) {
    uint4* q = reinterpret_cast<uint4*>(reinterpret_cast<__half*>(p.C) + (long long)orow * p.ldc + nc);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint4 u;
      u.x = pack_f16x2(v[i * 8 + 0], v[i * 8 + 1]);
      u.y = pack_f16x2(v[i * 8 + 2], v[i * 8 + 3]);
      u.z = pack_f16x2(v[i * 8 + 4], v[i * 8 + 5]);
      u.w = pack_f16x2(v[i * 8 + 6], v[i * 8 + 7]);
      q[i] = u;
      if (e.amax_out) {
        const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __half22float2(h[j]);
          amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
        }
      }
    }
  } else {
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.C) + (long long)orow * p.ldc + nc;
    uint4* q = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint4 u;
      u.x = pack_bf16x2(v[i * 8 + 0], v[i * 8 + 1]);
      u.y = pack_bf16x2(v[i * 8 + 2], v[i * 8 + 3]);
      u.z = pack_bf16x2(v[i * 8 + 4], v[i * 8 + 5]);
      u.w = pack_bf16x2(v[i * 8 + 6], v[i * 8 + 7]);
      q[i] = u;
      if (e.amax_out) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(h[j]);
          amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
        }
      }
    }
  }
}

// RMSNorm over one 64-column head (v = dims 0..31, w = dims 32..63) with its group's gamma, then
// rotate_half RoPE on dims 0..31 (pairs i, i+16) at this row's position; fp32 throughout.
// Rotary embedding on for column group g (at most 8 groups carry it; table mode has none).
__device__ __forceinline__ bool qk_rope_on(const sa3_epilogue& e, int g) { return g < 8 && ((e.qk_rope_mask >> g) & 1u); }

// RoPE cos/sin row of output row m (clamped into [0, M) for the padding rows of the last tile) for the
// 64-column head at nc, loaded before the tile's accumulator is ready. Leaves cs untouched when the
// head's group has no rotary embedding.
__device__ __forceinline__ void qk_rope_prefetch(const sa3_epilogue& e, int m, int M, int nc, int N, float (&cs)[32]) {
  if (nc >= N || !qk_rope_on(e, nc / e.qk_group_width)) return;
  m = m < M ? m : M - 1;
  int pos = e.row_pos ? __ldg(e.row_pos + m) : (e.rows_per_batch > 0 ? m % e.rows_per_batch : 0);
  if (pos >= e.max_pos) pos = e.max_pos - 1;
  if (pos < 0) pos = 0;
  ldg_f32x32(e.cos_sin + (long long)pos * 32, cs);  // cos[0..15], sin[0..15]
}

// qk RMSNorm (gamma of the head's group) of one 64-column head held as v = dims 0..31, w = dims 32..63.
// Packed fp32 pairs (sm_100 f32x2 arithmetic): one instruction per two elements, each lane rounded as the scalar op.
__device__ __forceinline__ uint64_t epi_pk2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 epi_up2(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t epi_fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t epi_mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// v[i] *= x[i] * y[i] over 32 elements in pairs (the scalar order: the product x*y first).
__device__ __forceinline__ void mul_prod32(float (&v)[32], const float (&x)[32], const float (&y)[32]) {
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    const float2 r = epi_up2(epi_mul2(epi_pk2(v[i], v[i + 1]), epi_mul2(epi_pk2(x[i], x[i + 1]), epi_pk2(y[i], y[i + 1]))));
    v[i] = r.x;
    v[i + 1] = r.y;
  }
}

__device__ __forceinline__ void qk_norm64(const sa3_epilogue& e, int nc, float (&v)[32], float (&w)[32]) {
  const int g = nc / e.qk_group_width;
  const float* gam = nullptr;
  if (e.qk_gamma_table) {
    if (g < e.qk_table_groups) gam = e.qk_gamma_table + 64 * g;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (g == i) gam = e.qk_gamma[i];
  }
  if (gam) {
    // both gamma halves are requested before the reduction; the sum of squares runs as 4 chains
    float g_lo[32], g_hi[32];
    ldg_f32x32(gam, g_lo);
    ldg_f32x32(gam + 32, g_hi);
    // four chains of squares, (0, 1) over v and (2, 3) over w, as packed pairs
    uint64_t a01 = epi_pk2(0.f, 0.f), a23 = epi_pk2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
      const uint64_t pv = epi_pk2(v[i], v[i + 1]), pw = epi_pk2(w[i], w[i + 1]);
      a01 = epi_fma2(pv, pv, a01);
      a23 = epi_fma2(pw, pw, a23);
    }
    const float2 s01 = epi_up2(a01), s23 = epi_up2(a23);
    const float r = rsqrtf(((s01.x + s01.y) + (s23.x + s23.y)) * (1.f / 64.f) + e.qk_eps);
    float rr[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) rr[i] = r;
    mul_prod32(v, rr, g_lo);
    mul_prod32(w, rr, g_hi);
  }
}

// Rotary embedding of dims 0..31 of the head (pairs i, i + 16) with the cos/sin row cs, when the
// head's group has one.
__device__ __forceinline__ void qk_rope64(const sa3_epilogue& e, int nc, const float (&cs)[32], float (&v)[32]) {
  if (qk_rope_on(e, nc / e.qk_group_width)) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float a = v[i], b = v[i + 16];
      v[i] = fmaf(a, cs[i], -b * cs[16 + i]);
      v[i + 16] = fmaf(b, cs[i], a * cs[16 + i]);
    }
  }
}

__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

// Residual kinds into the fp32 stream through TMA: the residual of this warp's 32 rows x 32 columns
// comes in as two 32 x 16 boxes (one per 2 KB buffer), is combined in place with the accumulator
// chunk v (this thread's row) and leaves as two TMA stores. rb = this row's CFG batch.
// Loads of one chunk's residual (lane 0). The first chunk of a tile is issued before the tile's
// accumulator is ready, so its latency hides behind the main loop.
__device__ __forceinline__ void residual_tma_issue(StoreStage& st, int M, int nc, int row0) {
  if (row0 >= M) return;  // warp-uniform
  st.pending = 1;
  if ((threadIdx.x & 31) != 0) return;
  bulk_wait_read_all();  // the stores of the previous chunk have read both buffers
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    mbar_arrive_expect_tx(&st.rbar[h], 2048);
    tma_load_2d(st.buf + h * 2048, st.tmr, &st.rbar[h], nc + 16 * h, row0);
  }
}

template <int KIND>
__device__ __forceinline__ void residual_tma_chunk(StoreStage& st, const GemmParams& p, int nc, int row0, int rb,
                                                   const float (&v)[32], float& amax) {
  const sa3_epilogue& e = p.epi;
  const int lane = threadIdx.x & 31;
  if (row0 >= p.M) return;  // warp-uniform: no valid row
  __syncwarp();
  const bool row_ok = row0 + lane < p.M;
  const int sw = (lane >> 1) & 3;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    mbar_wait(&st.rbar[h], st.uses & 1, st.abort, 77);
    if (h == 1) st.pending = 0;
    uint8_t* rowp = st.buf + h * 2048 + lane * 64;
    float4 g4[4];
    if (KIND == SA3_EPI_GATED_RESIDUAL) {
#pragma unroll
      for (int c = 0; c < 4; ++c)
        g4[c] = __ldg(reinterpret_cast<const float4*>(e.gate + (long long)rb * e.ld_gate + nc + 16 * h + 4 * c));
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float4* q = reinterpret_cast<float4*>(rowp + ((c ^ sw) * 16));
      float4 r = *q;
      const float* vv = v + 16 * h + 4 * c;
      if (KIND == SA3_EPI_GATED_RESIDUAL) {
        r.x = fmaf(vv[0], fast_sigmoid(1.f - g4[c].x), r.x);
        r.y = fmaf(vv[1], fast_sigmoid(1.f - g4[c].y), r.y);
        r.z = fmaf(vv[2], fast_sigmoid(1.f - g4[c].z), r.z);
        r.w = fmaf(vv[3], fast_sigmoid(1.f - g4[c].w), r.w);
      } else {
        r.x += vv[0];
        r.y += vv[1];
        r.z += vv[2];
        r.w += vv[3];
      }
      *q = r;
      if (e.amax_out && row_ok) amax = fmaxf(amax, fmaxf(fmaxf(fabsf(r.x), fabsf(r.y)), fmaxf(fabsf(r.z), fabsf(r.w))));
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(st.tm, st.buf + h * 2048, nc + 16 * h, row0);
      bulk_commit_group();
    }
  }
  st.uses++;
}

// In-place residual kinds (C is the residual): this warp's 32 rows x 32 columns of the branch output
// t = v (residual) or v * sigmoid(1 - gate[rb]) (gated) go through the two 2 KB buffers, in the 64-byte
// swizzle of the 16 x 32 fp32 box, and are added into C by two TMA reduce-adds. The stream is never
// loaded into the SM. A buffer is rewritten only after the reduce that last read it has read it.
template <int KIND>
__device__ __forceinline__ void residual_reduce_chunk(StoreStage& st, const GemmParams& p, int nc, int row0, int rb,
                                                      float (&v)[32]) {
  const sa3_epilogue& e = p.epi;
  const int lane = threadIdx.x & 31;
  if (row0 >= p.M) return;  // warp-uniform: no valid row
  if (KIND == SA3_EPI_GATED_RESIDUAL) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const float4 g = __ldg(reinterpret_cast<const float4*>(e.gate + (long long)rb * e.ld_gate + nc + 4 * c));
      v[4 * c] *= fast_sigmoid(1.f - g.x);
      v[4 * c + 1] *= fast_sigmoid(1.f - g.y);
      v[4 * c + 2] *= fast_sigmoid(1.f - g.z);
      v[4 * c + 3] *= fast_sigmoid(1.f - g.w);
    }
  }
  const int sw = (lane >> 1) & 3;
  if (st.f16) {
    // fp16 stream: this thread's 32 columns as fp16 in one 64-byte row of a 32 x 32 box, added by the L2
    uint8_t* b = st.buf + st.next * 2048;
    if (lane == 0) bulk_wait_read_all_but_one();  // the reduce issued two chunks ago has read this buffer
    __syncwarp();
    uint32_t w[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) w[i] = pack_f16x2(v[2 * i], v[2 * i + 1]);
#pragma unroll
    for (int c = 0; c < 4; ++c)
      *reinterpret_cast<uint4*>(b + lane * 64 + ((c ^ sw) * 16)) = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_reduce_add_2d(st.tm, b, nc, row0);
      bulk_commit_group();
    }
    st.next ^= 1;
    return;
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    if (lane == 0) bulk_wait_read_all_but_one();
    __syncwarp();
    uint8_t* rowp = st.buf + h * 2048 + lane * 64;
#pragma unroll
    for (int c = 0; c < 4; ++c)
      *reinterpret_cast<float4*>(rowp + ((c ^ sw) * 16)) =
          make_float4(v[16 * h + 4 * c], v[16 * h + 4 * c + 1], v[16 * h + 4 * c + 2], v[16 * h + 4 * c + 3]);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_reduce_add_2d(st.tm, st.buf + h * 2048, nc + 16 * h, row0);
      bulk_commit_group();
    }
  }
}

// Residual epilogues into the fp32 stream, transposed through a per-warp shared-memory scratch of
// 32 x 33 floats. TMEM hands each thread one row. In the write-back pass 8 threads cover one row's
// 32 columns with float4 accesses, so each warp instruction moves 4 full 128-byte row segments
// instead of 32 rows x 16 bytes. Thread t handles rows (t / 8) + 4k, k = 0..7, columns 4 (t % 8) ..
// +3; with the 33-float pitch both the row writes and these reads are free of bank conflicts. The
// output-row map and CFG batch of a row are computed once per tile by the lane that owns the row
// and handed out by shuffles. C may alias the residual: each element is read before the same
// thread writes it. Needs 16-byte aligned residual / C rows (the caller checks).
template <int KIND>
__device__ __forceinline__ void pg_residual_tile_t(const GemmParams& p, uint32_t tmem_tile, int m0, int n0, int q,
                                                   int half, float sa, float& amax, float* scratch) {
  const sa3_epilogue& e = p.epi;
  const int lane = threadIdx.x & 31;
  const uint32_t trow = tmem_tile + ((uint32_t)(q * 32) << 16);
  const int row0 = m0 + q * 32;
  const int nrows = min(32, p.M - row0);  // warp-uniform
  const float* res = reinterpret_cast<const float*>(e.residual);
  float* out = reinterpret_cast<float*>(p.C);
  const bool my_ok = lane < nrows;
  const int my_orow = my_ok ? out_row_of(e, row0 + lane) : 0;
  int my_batch = 0;
  if (KIND == SA3_EPI_GATED_RESIDUAL && my_ok)
    my_batch = e.row_batch ? __ldg(e.row_batch + row0 + lane) : (row0 + lane) / e.rows_per_batch;
  const int rsub = lane >> 3, c4 = 4 * (lane & 7);
  long long roff[8], ooff[8];
  int bk[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int orow = __shfl_sync(0xffffffffu, my_orow, rsub + 4 * k);
    roff[k] = (long long)orow * e.ld_residual;
    ooff[k] = (long long)orow * p.ldc;
    bk[k] = __shfl_sync(0xffffffffu, my_batch, rsub + 4 * k);
  }
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    const int col = half * 128 + c * 32;
    const int nc = n0 + col;
    if (nc >= p.N) break;  // uniform per warp
    float v[32];
    tmem_ld32(trow + col, v);
    scale_bias32(v, nc, sa, p.b_scale, e.bias);
#pragma unroll
    for (int i = 0; i < 32; ++i) scratch[lane * 33 + i] = v[i];
    __syncwarp();
    float4 r[8];
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (rsub + 4 * k < nrows) r[k] = *reinterpret_cast<const float4*>(res + roff[k] + nc + c4);  // may alias C
    int cur_b = -1;
    float4 gs = make_float4(1.f, 1.f, 1.f, 1.f);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int rr = rsub + 4 * k;
      if (rr < nrows) {
        const float* sp = scratch + rr * 33 + c4;
        float4 val = make_float4(sp[0], sp[1], sp[2], sp[3]);
        if (KIND == SA3_EPI_GATED_RESIDUAL) {
          if (bk[k] != cur_b) {
            cur_b = bk[k];
            const float4 g = __ldg(reinterpret_cast<const float4*>(e.gate + (long long)cur_b * e.ld_gate + nc + c4));
            gs = make_float4(fast_sigmoid(1.f - g.x), fast_sigmoid(1.f - g.y), fast_sigmoid(1.f - g.z),
                             fast_sigmoid(1.f - g.w));
          }
          val = make_float4(fmaf(val.x, gs.x, r[k].x), fmaf(val.y, gs.y, r[k].y), fmaf(val.z, gs.z, r[k].z),
                            fmaf(val.w, gs.w, r[k].w));
        } else {
          val = make_float4(val.x + r[k].x, val.y + r[k].y, val.z + r[k].z, val.w + r[k].w);
        }
        *reinterpret_cast<float4*>(out + ooff[k] + nc + c4) = val;
        if (e.amax_out) amax = fmaxf(amax, fmaxf(fmaxf(fabsf(val.x), fabsf(val.y)), fmaxf(fabsf(val.z), fabsf(val.w))));
      }
    }
    __syncwarp();
  }
}

// Epilogue of one 128 x 256 accumulator tile for the 32 rows of TMEM lane quarter q and column
// half `half` (tmem_tile = the tile's first TMEM column). Shared by the FP8/bf16 and GPTQ kernels.
// CS_PRE: for the qk-norm kind, *cs_pre is the cos/sin row of this thread's row, prefetched by
// qk_rope_prefetch for column n0 + half * 128 (all heads of a half belong to one group); otherwise it
// is loaded here per head.
template <int KIND, bool CS_PRE = false>
__device__ __forceinline__ void pg_epilogue_tile(const GemmParams& p, uint32_t tmem_tile, int m0, int n0, int q,
                                                 int half, float sa, float& amax, float* scratch = nullptr,
                                                 StoreStage* stg = nullptr, const float (*cs_pre)[32] = nullptr) {
  const sa3_epilogue& e = p.epi;
  const int lane = threadIdx.x & 31;
  if ((KIND == SA3_EPI_GATED_RESIDUAL || KIND == SA3_EPI_RESIDUAL) && stg && stg->red) {
    const uint32_t trow = tmem_tile + ((uint32_t)(q * 32) << 16);
    const int m = m0 + q * 32 + lane;
    int rb = 0;
    if (KIND == SA3_EPI_GATED_RESIDUAL && m < p.M) rb = e.row_batch ? __ldg(e.row_batch + m) : m / e.rows_per_batch;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      const int nc = n0 + half * 128 + c * 32;
      if (nc >= p.N) break;  // uniform per warp
      float v[32];
      tmem_ld32(trow + half * 128 + c * 32, v);
      scale_bias32(v, nc, sa, p.b_scale, e.bias);
      residual_reduce_chunk<KIND>(*stg, p, nc, m0 + q * 32, rb, v);
    }
    return;
  }
  if ((KIND == SA3_EPI_GATED_RESIDUAL || KIND == SA3_EPI_RESIDUAL) && stg && stg->tmr) {
    const uint32_t trow = tmem_tile + ((uint32_t)(q * 32) << 16);
    const int m = m0 + q * 32 + lane;
    int rb = 0;
    if (KIND == SA3_EPI_GATED_RESIDUAL && m < p.M) rb = e.row_batch ? __ldg(e.row_batch + m) : m / e.rows_per_batch;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      const int nc = n0 + half * 128 + c * 32;
      if (nc >= p.N) break;  // uniform per warp
      if (c > 0) residual_tma_issue(*stg, p.M, nc, m0 + q * 32);  // chunk 0 was issued by the caller
      float v[32];
      tmem_ld32(trow + half * 128 + c * 32, v);
      scale_bias32(v, nc, sa, p.b_scale, e.bias);
      residual_tma_chunk<KIND>(*stg, p, nc, m0 + q * 32, rb, v, amax);
    }
    return;
  }
  if ((KIND == SA3_EPI_GATED_RESIDUAL || KIND == SA3_EPI_RESIDUAL) && scratch && e.c_f32 &&
      ((reinterpret_cast<uintptr_t>(e.residual) | reinterpret_cast<uintptr_t>(p.C)) & 15) == 0 &&
      ((e.ld_residual | p.ldc) & 3) == 0 && (KIND != SA3_EPI_GATED_RESIDUAL || ((reinterpret_cast<uintptr_t>(e.gate) & 15) == 0 && (e.ld_gate & 3) == 0))) {
    pg_residual_tile_t<KIND>(p, tmem_tile, m0, n0, q, half, sa, amax, scratch);
    return;
  }
      const int m = m0 + q * 32 + lane;
      const int orow = out_row_of(e, m < p.M ? m : p.M - 1);
      int batch = 0;
      if (KIND == SA3_EPI_GATED_RESIDUAL && m < p.M)
        batch = e.row_batch ? __ldg(e.row_batch + m) : m / e.rows_per_batch;
      const uint32_t trow = tmem_tile + ((uint32_t)(q * 32) << 16);
      if (KIND == SA3_EPI_SWIGLU) {
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          const int col = half * 64 + c * 32;
          float x[32], g[32];
          tmem_ld32(trow + col, x);
          tmem_ld32(trow + 128 + col, g);
          scale_bias32(x, n0 + col, sa, p.b_scale, e.bias);
          scale_bias32(g, n0 + 128 + col, sa, p.b_scale, e.bias);
#pragma unroll
          for (int i = 0; i < 32; ++i) x[i] = x[i] * g[i] * fast_sigmoid(g[i]);
          if (stg)
            stage_store32(*stg, n0 / 2 + col, m0 + q * 32, p.M, x, amax, e.amax_out != nullptr);
          else
            pg_store_chunk<SA3_EPI_STORE>(p, m, orow, 0, n0 / 2 + col, x, amax);
        }
      } else if (KIND == SA3_EPI_QK_NORM) {
#pragma unroll 1
        for (int hh = 0; hh < 2; ++hh) {
          const int col = half * 128 + hh * 64;
          const int nc = n0 + col;
          if (nc >= p.N) break;  // uniform per warp
          float v[32], w[32];
          tmem_ld64(trow + col, v, w);  // both halves of the head under one wait
          if (p.b_scale && !e.bias) {
            // acc * (sa * b_scale[n]) in packed pairs, the scalar path's order
            float s[32], sa32[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) sa32[i] = sa;
            ldg_f32x32(p.b_scale + nc, s);
            mul_prod32(v, sa32, s);
            ldg_f32x32(p.b_scale + nc + 32, s);
            mul_prod32(w, sa32, s);
          } else {
            scale_bias32(v, nc, sa, p.b_scale, e.bias);
            scale_bias32(w, nc + 32, sa, p.b_scale, e.bias);
          }
          qk_norm64(e, nc, v, w);
          if (CS_PRE) {
            qk_rope64(e, nc, *cs_pre, v);
          } else if (qk_rope_on(e, nc / e.qk_group_width)) {
            float cs[32];  // the kernels with fewer registers per thread load it per head
            qk_rope_prefetch(e, m, p.M, nc, p.N, cs);
            qk_rope64(e, nc, cs, v);
          }
          if (stg) {
            stage_store32(*stg, nc, m0 + q * 32, p.M, v, amax, e.amax_out != nullptr);
            stage_store32(*stg, nc + 32, m0 + q * 32, p.M, w, amax, e.amax_out != nullptr);
          } else {
            pg_store_chunk<SA3_EPI_STORE>(p, m, orow, 0, nc, v, amax);
            pg_store_chunk<SA3_EPI_STORE>(p, m, orow, 0, nc + 32, w, amax);
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          const int col = half * 128 + c * 32;
          const int nc = n0 + col;
          if (nc >= p.N) break;  // uniform per warp
          float v[32];
          tmem_ld32(trow + col, v);
          scale_bias32(v, nc, sa, p.b_scale, e.bias);
          if ((KIND == SA3_EPI_STORE || KIND == SA3_EPI_SILU) && stg) {
            if (KIND == SA3_EPI_SILU) {
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = v[i] * fast_sigmoid(v[i]);
            }
            stage_store32(*stg, nc, m0 + q * 32, p.M, v, amax, e.amax_out != nullptr);
          } else {
            pg_store_chunk<KIND>(p, m, orow, batch, nc, v, amax);
          }
        }
      }
}

template <bool FP8, int KIND>
__global__ void __launch_bounds__(PG_THREADS, 1)
    gemm_persistent_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                           const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmR,
                           GemmParams p, int tiles_n, int num_tiles) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + GEMM_STAGES * GEMM_STAGE_BYTES);
  uint64_t* empty = full + GEMM_STAGES;
  uint64_t* acc_full = empty + GEMM_STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;        // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr int BK = FP8 ? 128 : 64;
  const int nkb = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < GEMM_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], PG_EPI_WARPS);
    }
    *abort_flag = 0;
    {
      uint64_t* rb = reinterpret_cast<uint64_t*>(smem + PG_SCRATCH_OFFSET + pg_rbar_offset());
      for (int i = 0; i < 2 * PG_EPI_WARPS; ++i) mbar_init(&rb[i], 1);
    }
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, PG_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dep_wait();  // the set-up above may run while the previous kernel on the stream retires

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
        const int m0 = (t / tiles_n) * GEMM_BM;
        const int n0 = (t % tiles_n) * GEMM_BN;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % GEMM_STAGES;
          if (it >= (uint32_t)GEMM_STAGES &&
              !mbar_wait(&empty[s], ((it / GEMM_STAGES) - 1) & 1, abort_flag, 31))
            break;
          uint8_t* st = smem + s * GEMM_STAGE_BYTES;
          mbar_arrive_expect_tx(&full[s], GEMM_STAGE_BYTES);
          tma_load_2d(st, &tmA, &full[s], kb * BK, m0);
          tma_load_2d(st + GEMM_A_BYTES, &tmB, &full[s], kb * BK, n0);
        }
      }
      if (*abort_flag) {
        // Drain this thread's loads that may still be in flight before the CTA exits.
        volatile int never = 0;
        const uint32_t first = it > (uint32_t)GEMM_STAGES ? it - GEMM_STAGES : 0;
        for (uint32_t j = first; j < it; ++j) mbar_wait(&full[j % GEMM_STAGES], (j / GEMM_STAGES) & 1, &never, 34);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = make_idesc(GEMM_BM, GEMM_BN, FP8 ? 0 : 1, FP8 ? 0 : 1, 0, 0);
      uint32_t it = 0, lt = 0;
      for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x, ++lt) {
        const uint32_t a = lt & 1;
        if (lt >= 2 && !mbar_wait(&acc_empty[a], ((lt >> 1) - 1) & 1, abort_flag, 32)) break;
        tc_fence_after();
        const uint32_t d = tmem + a * GEMM_BN;
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % GEMM_STAGES;
          if (!mbar_wait(&full[s], (it / GEMM_STAGES) & 1, abort_flag, 33)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * GEMM_STAGE_BYTES);
          const uint64_t ad = sdesc_kmajor_sw128(a_addr);
          const uint64_t bd = sdesc_kmajor_sw128(a_addr + GEMM_A_BYTES);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            if (FP8)
              mma_f8_ss(d, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
            else
              mma_f16_ss(d, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
          }
          tc_commit(&empty[s]);
        }
        tc_commit(&acc_full[a]);
        if (!ok) break;
      }
      // after an abort the epilogue may not wait for every accumulator: TMEM is released only once the
      // last commit on empty[] (it covers every MMA issued) has landed
      if (it > 0) {
        volatile int never = 0;
        mbar_wait(&empty[(it - 1) % GEMM_STAGES], ((it - 1) / GEMM_STAGES) & 1, &never, 36);
      }
    }
  } else {
    // ---------------- epilogue warps
    const int q = warp & 3;          // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;  // column half of the tile
    float* epi_scratch = reinterpret_cast<float*>(smem + PG_SCRATCH_OFFSET) + (warp - 2) * (32 * 33);
    // bf16 TMA-store staging reuses the same region with 512-byte aligned 2 x 2 KB buffers per warp
    uint64_t* rbars = reinterpret_cast<uint64_t*>(smem + PG_SCRATCH_OFFSET + pg_rbar_offset());
    StoreStage stg{&tmC, p.tma_store == 2 ? &tmR : nullptr, smem + ((PG_SCRATCH_OFFSET + 511) & ~511) + (warp - 2) * 4096,
                   rbars + 2 * (warp - 2), abort_flag, 0, 0, 0, p.tma_store == 3, p.epi.c_f16};
    StoreStage* stgp = p.tma_store ? &stg : nullptr;
    const sa3_epilogue& e = p.epi;
    const float sa = p.a_scale ? __ldg(p.a_scale) : 1.f;
    float amax = 0.f;
    uint32_t lt = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++lt) {
      const uint32_t a = lt & 1;
      const int m0 = (t / tiles_n) * GEMM_BM;
      const int n0 = (t % tiles_n) * GEMM_BN;
      if (stgp && stgp->tmr && n0 + half * 128 < p.N) residual_tma_issue(stg, p.M, n0 + half * 128, m0 + q * 32);
      if (!mbar_wait(&acc_full[a], (lt >> 1) & 1, abort_flag, 35)) break;
      tc_fence_after();
      pg_epilogue_tile<KIND>(p, tmem + a * GEMM_BN, m0, n0, q, half, sa, amax, epi_scratch, stgp);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
    }
    if (stgp && stg.pending) {
      // a residual load issued before an aborted accumulator wait: let it land before the CTA exits
      volatile int never = 0;
      mbar_wait(&stg.rbar[0], stg.uses & 1, &never, 78);
      mbar_wait(&stg.rbar[1], stg.uses & 1, &never, 78);
    }
    if (stgp && lane == 0) bulk_wait_all();  // this warp's TMA stores are complete before the CTA exits
    if (e.amax_out) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      if (lane == 0) atomic_max_nonneg(e.amax_out, amax);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, PG_TMEM_COLS);
}

// ---------------------------------------------------------------- 2-SM persistent GEMM
// A cluster of two CTAs (one per SM) computes 256 x 256 output tiles with tcgen05.mma.cta_group::2:
// CTA rank r holds A rows [m0 + 128 r, +128) and B rows [n0 + 128 r, +128) of every K slice, the
// leader (rank 0) issues M=256 N=256 MMAs that read both CTAs' shared memory, and each CTA's TMEM
// receives its own 128 x 256 accumulator. Per SM and K slice that is half the B bytes of the
// single-SM 128 x 256 tile, which is what lets the FP8 MMA run near its rate without exceeding the
// shared-memory bandwidth.
//   warp 0 (lane 0)  TMA of this CTA's A and B halves; both CTAs' copies complete on the leader's
//                    full barrier (the leader expects the bytes of both).
//   warp 1           leader: MMA issue (elected lane of the converged warp); commits signal the
//                    empty / acc_full barriers of both CTAs. Both CTAs: 2-SM TMEM allocation.
//   warps 2..9       epilogue of this CTA's 128 rows; the peer's warps report a drained
//                    accumulator on the leader's acc_empty barrier.
// All cluster-wide waits are bounded mbarrier waits except the two cluster barriers (after set-up
// and before exit), which every thread of both CTAs reaches on every path.
constexpr int P2_STAGES = 6;
constexpr int SA3_PAIR_MIN_ROWS = 512;  // below this the single-SM kernel has enough tiles to fill the GPU
constexpr int P2_A_BYTES = 128 * 128;  // 128 rows x 128-byte K slice
constexpr int P2_B_BYTES = 128 * 128;  // this CTA's half of the 256 B rows
constexpr int P2_STAGE_BYTES = P2_A_BYTES + P2_B_BYTES;
constexpr int P2_SCRATCH_OFFSET = P2_STAGES * P2_STAGE_BYTES + 256;
constexpr int P2_SMEM = P2_SCRATCH_OFFSET + PG_SCRATCH_BYTES + PG_RBAR_BYTES + 1024;
static_assert(P2_SCRATCH_OFFSET % 8 == 0, "mbarriers need 8-byte alignment");
static_assert(P2_SMEM <= 232448, "2-SM GEMM exceeds the 227 KB shared-memory limit");

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory object in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(addr), "r"(rank));
  return d;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// 2-D TMA load into this CTA's shared memory whose completion is counted on a barrier of the CTA
// pair (cluster address). No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* m, uint32_t bar_cluster, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}
template <bool FP8>
__device__ __forceinline__ void mma_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  if (FP8)
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t.reg .b32 r;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "elect.sync r|e, 0xffffffff;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  else
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t.reg .b32 r;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "elect.sync r|e, 0xffffffff;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on the barrier at this offset in both CTAs once the pair MMAs issued so far are done.
__device__ __forceinline__ void commit_pair_both(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t.reg .b32 r;\n\t.reg .b16 m;\n\t"
      "mov.b16 m, 3;\n\t"
      "elect.sync r|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}\n" ::"r"(
          smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
__device__ __forceinline__ bool warp_wait_g(uint64_t* bar, uint32_t parity, volatile int* abort, int site) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, site));
}

template <bool FP8, int KIND>
__global__ void __launch_bounds__(PG_THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmR,
                     GemmParams p, int tiles_n, int num_tiles) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + P2_STAGES * P2_STAGE_BYTES);
  uint64_t* empty = full + P2_STAGES;
  uint64_t* acc_full = empty + P2_STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;      // [2], leader only: 2 x PG_EPI_WARPS arrivals
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  constexpr int BK = FP8 ? 128 : 64;
  const int nkb = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P2_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 2 * PG_EPI_WARPS);
    }
    *abort_flag = 0;
    {
      uint64_t* rb = reinterpret_cast<uint64_t*>(smem + P2_SCRATCH_OFFSET + pg_rbar_offset());
      for (int i = 0; i < 2 * PG_EPI_WARPS; ++i) mbar_init(&rb[i], 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(PG_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated in both
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dep_wait();  // the set-up above may run while the previous kernel on the stream retires

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      for (int t = pair; t < num_tiles && !*abort_flag; t += npairs) {
        const int m0 = (t / tiles_n) * 256 + 128 * (int)rank;
        const int n0 = (t % tiles_n) * 256 + 128 * (int)rank;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % P2_STAGES;
          if (it >= (uint32_t)P2_STAGES && !mbar_wait(&empty[s], ((it / P2_STAGES) - 1) & 1, abort_flag, 71)) break;
          uint8_t* st = smem + s * P2_STAGE_BYTES;
          const uint32_t fbar = mapa_shared(smem_u32(&full[s]), 0);
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * P2_STAGE_BYTES);
          tma_load_2d_pair(st, &tmA, fbar, kb * BK, m0);
          tma_load_2d_pair(st + P2_A_BYTES, &tmB, fbar, kb * BK, n0);
        }
      }
      if (*abort_flag && rank == 0) {
        // both CTAs' copies complete on the leader's barriers: wait (bounded) for the last ones
        volatile int never = 0;
        const uint32_t first = it > (uint32_t)P2_STAGES ? it - P2_STAGES : 0;
        for (uint32_t j = first; j < it; ++j) mbar_wait(&full[j % P2_STAGES], (j / P2_STAGES) & 1, &never, 72);
      }
    }
  } else if (warp == 1) {
    if (rank == 0) {
      // the instruction descriptor takes M = 256 for the pair
      const uint32_t idesc = make_idesc(256, 256, FP8 ? 0 : 1, FP8 ? 0 : 1, 0, 0);
      uint32_t it = 0, lt = 0;
      bool ok = true;
      for (int t = pair; t < num_tiles && ok; t += npairs, ++lt) {
        const uint32_t a = lt & 1;
        if (lt >= 2 && !warp_wait_g(&acc_empty[a], ((lt >> 1) - 1) & 1, abort_flag, 73)) break;
        tc_fence_after();
        const uint32_t d = tmem + a * GEMM_BN;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % P2_STAGES;
          if (!warp_wait_g(&full[s], (it / P2_STAGES) & 1, abort_flag, 74)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * P2_STAGE_BYTES);
          const uint64_t ad = sdesc_kmajor_sw128(a_addr);
          const uint64_t bd = sdesc_kmajor_sw128(a_addr + P2_A_BYTES);
#pragma unroll
          for (int k = 0; k < 4; ++k) mma_pair<FP8>(d, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
          commit_pair_both(&empty[s]);
        }
        commit_pair_both(&acc_full[a]);
      }
      // TMEM is released after the final cluster barrier: no MMA may still be running then. The last
      // commit on empty[] covers every MMA this thread issued, and nothing commits to that barrier
      // afterwards. (An extra commit on acc_full here would complete a second phase of a buffer whose
      // previous phase a lagging epilogue warp may not have observed yet; with a phase-parity wait that
      // warp would then wait for a phase that never comes.)
      if (it > 0) {
        volatile int never = 0;
        warp_wait_g(&empty[(it - 1) % P2_STAGES], ((it - 1) / P2_STAGES) & 1, &never, 75);
      }
    }
  } else {
    // ---------------- epilogue warps
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    float* epi_scratch = reinterpret_cast<float*>(smem + P2_SCRATCH_OFFSET) + (warp - 2) * (32 * 33);
    // bf16 TMA-store staging reuses the same region with 512-byte aligned 2 x 2 KB buffers per warp
    uint64_t* rbars = reinterpret_cast<uint64_t*>(smem + P2_SCRATCH_OFFSET + pg_rbar_offset());
    StoreStage stg{&tmC, p.tma_store == 2 ? &tmR : nullptr, smem + ((P2_SCRATCH_OFFSET + 511) & ~511) + (warp - 2) * 4096,
                   rbars + 2 * (warp - 2), abort_flag, 0, 0, 0, p.tma_store == 3, p.epi.c_f16};
    StoreStage* stgp = p.tma_store ? &stg : nullptr;
    const sa3_epilogue& e = p.epi;
    const float sa = p.a_scale ? __ldg(p.a_scale) : 1.f;
    float amax = 0.f;
    uint32_t lt = 0;
    for (int t = pair; t < num_tiles; t += npairs, ++lt) {
      const uint32_t a = lt & 1;
      const int m0 = (t / tiles_n) * 256 + 128 * (int)rank;
      const int n0 = (t % tiles_n) * 256;
      if (stgp && stgp->tmr && n0 + half * 128 < p.N) residual_tma_issue(stg, p.M, n0 + half * 128, m0 + q * 32);
      float cs[32];
      if (KIND == SA3_EPI_QK_NORM) qk_rope_prefetch(e, m0 + q * 32 + lane, p.M, n0 + half * 128, p.N, cs);
      if (!mbar_wait(&acc_full[a], (lt >> 1) & 1, abort_flag, 76)) break;
      tc_fence_after();
      pg_epilogue_tile<KIND, KIND == SA3_EPI_QK_NORM>(p, tmem + a * GEMM_BN, m0, n0, q, half, sa, amax, epi_scratch,
                                                       stgp, &cs);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0)
          mbar_arrive(&acc_empty[a]);
        else
          mbar_arrive_cluster(mapa_shared(smem_u32(&acc_empty[a]), 0));
      }
    }
    if (stgp && stg.pending) {
      // a residual load issued before an aborted accumulator wait: let it land before the CTA exits
      volatile int never = 0;
      mbar_wait(&stg.rbar[0], stg.uses & 1, &never, 78);
      mbar_wait(&stg.rbar[1], stg.uses & 1, &never, 78);
    }
    if (stgp && lane == 0) bulk_wait_all();  // this warp's TMA stores are complete before the CTA exits
    if (e.amax_out) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      if (lane == 0) atomic_max_nonneg(e.amax_out, amax);
    }
  }

  __syncwarp();  // reconverge the single-lane roles before the aligned cluster barrier
  tc_fence_before();
  cluster_sync_all();  // neither CTA leaves while the other may still touch its barriers or memory
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(PG_TMEM_COLS) : "memory");
  }
}

template <bool FP8>
static int launch_pair(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmC,
                       const CUtensorMap& tmR, const GemmParams& p, int kind, cudaStream_t st) {
  const int tiles_n = (p.N + 255) / 256;
  const int tiles_m = (p.M + 255) / 256;
  const int num_tiles = tiles_n * tiles_m;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 2)
    return SA3_ERR_LAUNCH;
  const int npairs = num_tiles < sms / 2 ? num_tiles : sms / 2;
  int rc;
#define SA3_P2_CASE(K)                                                                               \
  case K:                                                                                            \
    if ((rc = ensure_smem(gemm_pair_kernel<FP8, K>, P2_SMEM))) return rc;                            \
    if ((rc = launch_ex(gemm_pair_kernel<FP8, K>, dim3(2 * npairs), dim3(PG_THREADS), P2_SMEM, st, 2, tmA, tmB, \
                        tmC, tmR, p, tiles_n, num_tiles)))                                                  \
      return rc;                                                                                     \
    break;
  switch (kind) {
    SA3_P2_CASE(SA3_EPI_STORE)
    SA3_P2_CASE(SA3_EPI_SILU)
    SA3_P2_CASE(SA3_EPI_SWIGLU)
    SA3_P2_CASE(SA3_EPI_GATED_RESIDUAL)
    SA3_P2_CASE(SA3_EPI_RESIDUAL)
    SA3_P2_CASE(SA3_EPI_QK_NORM)
    default:
      return SA3_ERR_ARG;
  }
#undef SA3_P2_CASE
  return launch_status();
}

template <bool FP8>
static int launch_persistent(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmC,
                             const CUtensorMap& tmR, const GemmParams& p, int kind, cudaStream_t st) {
  const int tiles_n = (p.N + GEMM_BN - 1) / GEMM_BN;
  const int tiles_m = (p.M + GEMM_BM - 1) / GEMM_BM;
  const int num_tiles = tiles_n * tiles_m;
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  const int grid = num_tiles < sms ? num_tiles : sms;
  int rc;
#define SA3_PG_CASE(K)                                                                                   \
  case K:                                                                                                \
    if ((rc = ensure_smem(gemm_persistent_kernel<FP8, K>, PG_SMEM))) return rc;                          \
    launch_ex(gemm_persistent_kernel<FP8, K>, dim3(grid), dim3(PG_THREADS), PG_SMEM, st, 1, tmA, tmB, tmC, tmR, p, tiles_n, num_tiles); \
    break;
  switch (kind) {
    SA3_PG_CASE(SA3_EPI_STORE)
    SA3_PG_CASE(SA3_EPI_SILU)
    SA3_PG_CASE(SA3_EPI_SWIGLU)
    SA3_PG_CASE(SA3_EPI_GATED_RESIDUAL)
    SA3_PG_CASE(SA3_EPI_RESIDUAL)
    SA3_PG_CASE(SA3_EPI_QK_NORM)
    default:
      return SA3_ERR_ARG;
  }
#undef SA3_PG_CASE
  return launch_status();
}


// ---------------------------------------------------------------------------------------------
// GPTQ int4 weight-only GEMM: C = epilogue(A . W^T), A bf16 [M, K] (input channels already in
// group-sorted act-order), W given as
//   qw  int32 [N, K/8]  : word (n, w) holds q[n, k] for k = 8w + j in bits [4j, 4j+4)
//   sz  fp32  [G, 2N]   : row g = [ s[g, 0..N) | z*s[g, 0..N) ], group g covers k in [g*gs, (g+1)*gs)
// W[n, k] = q*s - z*s = (q - z) * s (exact in fp32), rounded once to bf16 in shared memory.
// Persistent, 14 warps: warp 0 TMA (A tile, packed W tile, s and z*s rows), warp 1 tcgen05.mma
// (kind::f16, bf16), warps 2..5 epilogue (TMEM double buffer), warps 6..13 dequantise the packed
// tile into a 128-byte-swizzled K-major bf16 B tile.
constexpr int GQ_STAGES = 3;
constexpr int GQ_A_BYTES = 16384;   // 128 x 64 bf16
constexpr int GQ_BD_BYTES = 32768;  // 256 x 64 bf16 (dequantised)
constexpr int GQ_BP_BYTES = 8192;   // 256 x 8 packed words
constexpr int GQ_SZ_BYTES = 2048;   // 256 s + 256 z*s
constexpr int GQ_STAGE_BYTES = GQ_A_BYTES + GQ_BD_BYTES + GQ_BP_BYTES + GQ_SZ_BYTES;
constexpr int GQ_THREADS = 448;
constexpr int GQ_SMEM = GQ_STAGES * GQ_STAGE_BYTES + 1024 + 256;

__device__ __forceinline__ uint4 gptq_dequant8(uint32_t word, float sc, float zs) {
  float w[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t q = (word >> (4 * j)) & 0xFu;
    const float f = __uint_as_float(0x4B000000u | q) - 8388608.f;  // exact float(q)
    w[j] = fmaf(f, sc, -zs);                                        // (q - z) * s, exact
  }
  uint4 u;
  u.x = pack_bf16x2(w[0], w[1]);
  u.y = pack_bf16x2(w[2], w[3]);
  u.z = pack_bf16x2(w[4], w[5]);
  u.w = pack_bf16x2(w[6], w[7]);
  return u;
}

template <int KIND>
__global__ void __launch_bounds__(GQ_THREADS, 1)
    gemm_gptq_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                     const __grid_constant__ CUtensorMap tmSZ, GemmParams p, int tiles_n, int num_tiles,
                     int group_size) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + GQ_STAGES * GQ_STAGE_BYTES);
  uint64_t* dq = full + GQ_STAGES;
  uint64_t* empty = dq + GQ_STAGES;
  uint64_t* acc_full = empty + GQ_STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
#define GQ_A(s) (smem + (s) * GQ_STAGE_BYTES)
#define GQ_BD(s) (smem + (s) * GQ_STAGE_BYTES + GQ_A_BYTES)
#define GQ_BP(s) (smem + (s) * GQ_STAGE_BYTES + GQ_A_BYTES + GQ_BD_BYTES)
#define GQ_SZ(s) (smem + (s) * GQ_STAGE_BYTES + GQ_A_BYTES + GQ_BD_BYTES + GQ_BP_BYTES)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = p.K / 64;
  if (threadIdx.x == 0) {
    for (int i = 0; i < GQ_STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&dq[i], 8);
      mbar_init(&empty[i], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmSZ);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, PG_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dep_wait();  // the set-up above may run while the previous kernel on the stream retires

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
        const int m0 = (t / tiles_n) * GEMM_BM;
        const int n0 = (t % tiles_n) * GEMM_BN;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % GQ_STAGES;
          if (it >= (uint32_t)GQ_STAGES && !mbar_wait(&empty[s], ((it / GQ_STAGES) - 1) & 1, abort_flag, 51)) break;
          const int g = (kb * 64) / group_size;
          mbar_arrive_expect_tx(&full[s], GQ_A_BYTES + GQ_BP_BYTES + GQ_SZ_BYTES);
          tma_load_2d(GQ_A(s), &tmA, &full[s], kb * 64, m0);
          tma_load_2d(GQ_BP(s), &tmW, &full[s], kb * 8, n0);
          tma_load_2d(GQ_SZ(s), &tmSZ, &full[s], n0, g);
          tma_load_2d(GQ_SZ(s) + 1024, &tmSZ, &full[s], p.N + n0, g);
        }
      }
      if (*abort_flag) {
        volatile int never = 0;
        // the last GQ_STAGES issued stages are the only ones that can still be in flight
        for (int s = 0; s < GQ_STAGES; ++s) mbar_wait(&full[s], 0, &never, 52);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = make_idesc(GEMM_BM, GEMM_BN, 1, 1, 0, 0);
      uint32_t it = 0, lt = 0;
      for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x, ++lt) {
        const uint32_t a = lt & 1;
        if (lt >= 2 && !mbar_wait(&acc_empty[a], ((lt >> 1) - 1) & 1, abort_flag, 53)) break;
        tc_fence_after();
        const uint32_t d = tmem + a * GEMM_BN;
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % GQ_STAGES;
          if (!mbar_wait(&dq[s], (it / GQ_STAGES) & 1, abort_flag, 54)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sdesc_kmajor_sw128(smem_u32(GQ_A(s)));
          const uint64_t bd = sdesc_kmajor_sw128(smem_u32(GQ_BD(s)));
#pragma unroll
          for (int k = 0; k < 4; ++k) mma_f16_ss(d, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
          tc_commit(&empty[s]);
        }
        tc_commit(&acc_full[a]);
        if (!ok) break;
      }
      // TMEM is released only once the last commit on empty[] (it covers every MMA issued) has landed
      if (it > 0) {
        volatile int never = 0;
        mbar_wait(&empty[(it - 1) % GQ_STAGES], ((it - 1) / GQ_STAGES) & 1, &never, 57);
      }
    }
  } else if (warp < 6) {
    const int q = warp & 3;
    float amax = 0.f;
    uint32_t lt = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++lt) {
      const uint32_t a = lt & 1;
      if (!mbar_wait(&acc_full[a], (lt >> 1) & 1, abort_flag, 55)) break;
      tc_fence_after();
      const int m0 = (t / tiles_n) * GEMM_BM;
      const int n0 = (t % tiles_n) * GEMM_BN;
      pg_epilogue_tile<KIND>(p, tmem + a * GEMM_BN, m0, n0, q, 0, 1.f, amax);
      pg_epilogue_tile<KIND>(p, tmem + a * GEMM_BN, m0, n0, q, 1, 1.f, amax);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
    }
    if (p.epi.amax_out) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      if (lane == 0) atomic_max_nonneg(p.epi.amax_out, amax);
    }
  } else {
    // ---------------- dequantisation warps: thread t handles words t + 256 i (n = word / 8, w = word % 8)
    const int t = (warp - 6) * 32 + lane;
    uint32_t it = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = it % GQ_STAGES;
        if (!mbar_wait(&full[s], (it / GQ_STAGES) & 1, abort_flag, 56)) break;
        const uint32_t* bp = reinterpret_cast<const uint32_t*>(GQ_BP(s));
        const float* sc = reinterpret_cast<const float*>(GQ_SZ(s));
        uint8_t* bd = GQ_BD(s);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int item = i * 256 + t;
          const int n = item >> 3, w = item & 7;
          const uint4 u = gptq_dequant8(bp[item], sc[n], sc[256 + n]);
          *reinterpret_cast<uint4*>(bd + n * 128 + ((w ^ (n & 7)) << 4)) = u;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&dq[s]);
      }
      if (*abort_flag) break;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, PG_TMEM_COLS);
#undef GQ_A
#undef GQ_BD
#undef GQ_BP
#undef GQ_SZ
}

__global__ void __launch_bounds__(256) gptq_dequant_kernel(const uint32_t* qw, const float* sz, __nv_bfloat16* out,
                                                           int N, int K, int group_size) {
  grid_dep_wait();
  const long long words = (long long)N * (K / 8);
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < words; i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i / (K / 8));
    const int w = (int)(i - (long long)n * (K / 8));
    const int g = (w * 8) / group_size;
    const uint4 u = gptq_dequant8(qw[i], sz[(long long)g * 2 * N + n], sz[(long long)g * 2 * N + N + n]);
    *reinterpret_cast<uint4*>(out + (long long)n * K + w * 8) = u;
  }
}

// W [N, K] bf16 in the ORIGINAL input-channel order: W[n, k] is the weight of sorted position
// inv_perm[k]. One weight row per iteration: its K/8 packed words and its (s, z*s) pair of every group
// are staged in shared memory, then each thread writes 8 consecutive channels (one 16-byte store),
// gathering their nibbles through inv_perm. Same arithmetic as gptq_dequant8: fma(q, s, -z*s), exact in
// fp32, rounded once to bf16.
__global__ void __launch_bounds__(256) gptq_dequant_orig_kernel(const uint32_t* qw, const float* sz,
                                                                const int* inv_perm, __nv_bfloat16* out, int N,
                                                                int K, long long ldo, int group_size) {
  grid_dep_wait();
  extern __shared__ __align__(16) uint8_t dq_raw[];
  uint32_t* words = reinterpret_cast<uint32_t*>(dq_raw);  // K / 8
  float* ssz = reinterpret_cast<float*>(words + K / 8);   // [G][2]: s, z*s
  const int G = K / group_size;
  for (int n = blockIdx.x; n < N; n += gridDim.x) {
    for (int c = threadIdx.x; c < K / 8; c += blockDim.x) words[c] = __ldg(qw + (long long)n * (K / 8) + c);
    for (int g = threadIdx.x; g < G; g += blockDim.x) {
      ssz[2 * g] = __ldg(sz + (long long)g * 2 * N + n);
      ssz[2 * g + 1] = __ldg(sz + (long long)g * 2 * N + N + n);
    }
    __syncthreads();
    for (int c = threadIdx.x; c < K / 8; c += blockDim.x) {
      const int4 p0 = __ldg(reinterpret_cast<const int4*>(inv_perm) + 2 * c);
      const int4 p1 = __ldg(reinterpret_cast<const int4*>(inv_perm) + 2 * c + 1);
      const int sp[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
      float w[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t q = (words[sp[j] >> 3] >> (4 * (sp[j] & 7))) & 0xFu;
        const int g = sp[j] / group_size;
        const float f = __uint_as_float(0x4B000000u | q) - 8388608.f;  // exact float(q)
        w[j] = fmaf(f, ssz[2 * g], -ssz[2 * g + 1]);                    // (q - z) * s, exact
      }
      uint4 u;
      u.x = pack_bf16x2(w[0], w[1]);
      u.y = pack_bf16x2(w[2], w[3]);
      u.z = pack_bf16x2(w[4], w[5]);
      u.w = pack_bf16x2(w[6], w[7]);
      *reinterpret_cast<uint4*>(out + (long long)n * ldo + 8 * c) = u;
    }
    __syncthreads();
  }
}

// out[r, j] = x[r, perm[j]] (bf16); one row staged in shared memory per iteration.
__global__ void __launch_bounds__(256) permute_cols_kernel(const __nv_bfloat16* x, const int* perm, __nv_bfloat16* out,
                                                           int rows, int K, long long ldx, long long ldo) {
  grid_dep_wait();
  extern __shared__ __align__(16) uint8_t prow_raw[];
  __nv_bfloat16* rowbuf = reinterpret_cast<__nv_bfloat16*>(prow_raw);
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const uint4* src = reinterpret_cast<const uint4*>(x + (long long)r * ldx);
    for (int c = threadIdx.x; c < K / 8; c += blockDim.x) reinterpret_cast<uint4*>(rowbuf)[c] = src[c];
    __syncthreads();
    for (int c = threadIdx.x; c < K / 8; c += blockDim.x) {
      const int4 p0 = __ldg(reinterpret_cast<const int4*>(perm) + 2 * c);
      const int4 p1 = __ldg(reinterpret_cast<const int4*>(perm) + 2 * c + 1);
      __nv_bfloat162 h0, h1, h2, h3;
      h0.x = rowbuf[p0.x]; h0.y = rowbuf[p0.y];
      h1.x = rowbuf[p0.z]; h1.y = rowbuf[p0.w];
      h2.x = rowbuf[p1.x]; h2.y = rowbuf[p1.y];
      h3.x = rowbuf[p1.z]; h3.y = rowbuf[p1.w];
      uint4 u;
      u.x = *reinterpret_cast<uint32_t*>(&h0);
      u.y = *reinterpret_cast<uint32_t*>(&h1);
      u.z = *reinterpret_cast<uint32_t*>(&h2);
      u.w = *reinterpret_cast<uint32_t*>(&h3);
      reinterpret_cast<uint4*>(out + (long long)r * ldo)[c] = u;
    }
    __syncthreads();
  }
}

}  // namespace sa3

using namespace sa3;

extern "C" int sa3_version(void) { return 100; }

extern "C" int sa3_get_device_error(int* err) {
  if (!err) return SA3_ERR_ARG;
  if (cudaDeviceSynchronize() != cudaSuccess) return SA3_ERR_LAUNCH;
  int a = 0, b = 0, c = 0, d = 0, rc;
  if ((rc = read_error_gemm(&a)) || (rc = read_error_glue(&b)) || (rc = read_error_attention(&c)) ||
      (rc = read_error_peer(&d)))
    return rc;
  *err = a ? a : (b ? b : (c ? c : d));
  return SA3_OK;
}

extern "C" int sa3_gemm(const void* A, const void* B, void* C, int M, int N, int K, long long lda, long long ldb,
                        long long ldc, int ab_dtype, const float* a_scale, const float* b_scale,
                        const sa3_epilogue* epi, void* stream) {
  if (!A || !B || !C || M <= 0 || N <= 0 || K <= 0) return SA3_ERR_ARG;
  if (ab_dtype != SA3_DT_BF16 && ab_dtype != SA3_DT_E4M3) return SA3_ERR_DTYPE;
  const bool fp8 = ab_dtype == SA3_DT_E4M3;
  const int esz = fp8 ? 1 : 2;
  if (lda < K || ldb < K) return SA3_ERR_ARG;
  if (!aligned16(A) || !aligned16(B) || ((lda * esz) % 16) || ((ldb * esz) % 16)) return SA3_ERR_ALIGN;
  sa3_epilogue e{};
  if (epi) e = *epi;
  if (e.kind < SA3_EPI_STORE || e.kind > SA3_EPI_QK_NORM) return SA3_ERR_ARG;
  if (e.c_f32 && e.c_f16) return SA3_ERR_ARG;
  if (e.c_f16 && (e.kind == SA3_EPI_SWIGLU || e.kind == SA3_EPI_QK_NORM)) return SA3_ERR_UNSUPPORTED;
  if (e.kind == SA3_EPI_QK_NORM) {
    if (e.qk_group_width <= 0 || e.qk_group_width % 64) return SA3_ERR_ARG;
    if (e.qk_gamma_table) {
      if (e.qk_table_groups <= 0 || e.qk_rope_mask) return SA3_ERR_ARG;
      if (!aligned16(e.qk_gamma_table)) return SA3_ERR_ALIGN;
    } else if (N > 8 * e.qk_group_width) {
      return SA3_ERR_ARG;
    }
    for (int g = 0; g < 8; ++g)
      if (e.qk_gamma[g] && !aligned16(e.qk_gamma[g])) return SA3_ERR_ALIGN;
    if (e.qk_rope_mask && (!e.cos_sin || !aligned16(e.cos_sin) || e.max_pos <= 0 ||
                           (!e.row_pos && e.rows_per_batch <= 0)))
      return SA3_ERR_ARG;
  }
  if (e.kind == SA3_EPI_SWIGLU) {
    if (e.c_f32) return SA3_ERR_UNSUPPORTED;
    if (N % GEMM_BN != 0) return SA3_ERR_UNSUPPORTED;
    if (ldc < N / 2) return SA3_ERR_ARG;
  } else if (ldc < N) {
    return SA3_ERR_ARG;
  }
  if ((e.kind == SA3_EPI_GATED_RESIDUAL || e.kind == SA3_EPI_RESIDUAL) && !e.residual) return SA3_ERR_ARG;
  if (e.kind == SA3_EPI_GATED_RESIDUAL && !e.gate) return SA3_ERR_ARG;
  if (e.kind == SA3_EPI_GATED_RESIDUAL && !e.row_batch && e.rows_per_batch <= 0) return SA3_ERR_ARG;
  if (e.seg_in < 0 || (e.seg_in > 0 && e.seg_out <= 0)) return SA3_ERR_ARG;

  CUtensorMap tmA, tmB;
  const CUtensorMapDataType dt = fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint32_t bk = fp8 ? 128 : 64;
  int rc = make_tmap_2d(&tmA, A, dt, esz, (uint64_t)K, (uint64_t)M, (uint64_t)lda, bk, GEMM_BM);
  if (rc) return rc;
  rc = make_tmap_2d(&tmB, B, dt, esz, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, bk, GEMM_BN);
  if (rc) return rc;

  GemmParams p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.ldc = ldc;
  p.C = C;
  p.a_scale = a_scale;
  p.b_scale = b_scale;
  p.epi = e;

  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // Fast path: persistent kernel with an overlapped, vectorised epilogue.
  auto al16 = [](const void* q) { return q == nullptr || aligned16(q); };
  const bool res_kind = e.kind == SA3_EPI_GATED_RESIDUAL || e.kind == SA3_EPI_RESIDUAL;
  const int celt = e.c_f32 ? 4 : 2;
  bool fast = (N % 32 == 0) && aligned16(C) && ((ldc * celt) % 16 == 0) && al16(b_scale) && al16(e.bias) &&
              (e.kind != SA3_EPI_SWIGLU || N % GEMM_BN == 0);
  if (res_kind) fast = fast && aligned16(e.residual) && ((e.ld_residual * celt) % 16 == 0);
  if (e.kind == SA3_EPI_GATED_RESIDUAL) fast = fast && aligned16(e.gate) && (e.ld_gate % 4 == 0);
  if (!fast && (e.kind == SA3_EPI_QK_NORM || e.c_f16)) return SA3_ERR_UNSUPPORTED;  // only the persistent kernels
  // bf16 outputs without a row remap leave through TMA stores (tmC); otherwise tmC is unused
  CUtensorMap tmC = tmA;
  p.tma_store = 0;
  if (fast && !e.c_f32 && !e.c_f16 && !e.out_row_map && e.seg_in == 0 &&
      (e.kind == SA3_EPI_STORE || e.kind == SA3_EPI_SILU || e.kind == SA3_EPI_SWIGLU || e.kind == SA3_EPI_QK_NORM)) {
    const uint64_t ccols = e.kind == SA3_EPI_SWIGLU ? (uint64_t)N / 2 : (uint64_t)N;
    if ((rc = make_tmap_2d(&tmC, C, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ccols, (uint64_t)M, (uint64_t)ldc, 32, 32,
                           CU_TENSOR_MAP_SWIZZLE_64B)))
      return rc;
    p.tma_store = 1;
  }
  // fp32 residual kinds without a row remap: residual in and result out through TMA (tma_store = 2)
  CUtensorMap tmR = tmA;
  if (fast && e.c_f32 && !e.out_row_map && e.seg_in == 0 &&
      (e.kind == SA3_EPI_GATED_RESIDUAL || e.kind == SA3_EPI_RESIDUAL) && (e.kind != SA3_EPI_GATED_RESIDUAL || e.ld_gate % 4 == 0)) {
    if ((rc = make_tmap_2d(&tmC, C, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)N, (uint64_t)M, (uint64_t)ldc, 16, 32,
                           CU_TENSOR_MAP_SWIZZLE_64B)))
      return rc;
    if (e.residual == C && e.ld_residual == ldc && !e.amax_out && sa3_residual_reduce_enabled()) {
      p.tma_store = 3;  // in place and nothing needs the updated values: reduce-add into C
    } else {
      if ((rc = make_tmap_2d(&tmR, e.residual, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)N, (uint64_t)M,
                             (uint64_t)e.ld_residual, 16, 32, CU_TENSOR_MAP_SWIZZLE_64B)))
        return rc;
      p.tma_store = 2;
    }
  }
  // fp16 residual stream, in place: reduce-add of the fp16-rounded result into C (tma_store = 3 with an fp16 map of
  // 32 x 32 boxes, the bf16 store layout)
  if (fast && e.c_f16 && res_kind && !e.out_row_map && e.seg_in == 0 && e.residual == C && e.ld_residual == ldc &&
      !e.amax_out && sa3_residual_reduce_enabled()) {
    if ((rc = make_tmap_2d(&tmC, C, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)N, (uint64_t)M, (uint64_t)ldc, 32, 32,
                           CU_TENSOR_MAP_SWIZZLE_64B)))
      return rc;
    p.tma_store = 3;
  }
  if (fast && M >= SA3_PAIR_MIN_ROWS) {
    // enough rows for 256-row tiles: the 2-SM kernel (FP8 or bf16). Its A and B boxes are 128 rows.
    CUtensorMap tmB2;
    if ((rc = make_tmap_2d(&tmB2, B, dt, esz, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, bk, 128))) return rc;
    return fp8 ? launch_pair<true>(tmA, tmB2, tmC, tmR, p, e.kind, st)
               : launch_pair<false>(tmA, tmB2, tmC, tmR, p, e.kind, st);
  }
  if (fast)
    return fp8 ? launch_persistent<true>(tmA, tmB, tmC, tmR, p, e.kind, st)
               : launch_persistent<false>(tmA, tmB, tmC, tmR, p, e.kind, st);

  dim3 grid((N + GEMM_BN - 1) / GEMM_BN, (M + GEMM_BM - 1) / GEMM_BM);
  if (grid.y > 65535) return SA3_ERR_UNSUPPORTED;
  if (fp8) {
    if ((rc = ensure_smem(gemm_tc_kernel<true>, GEMM_SMEM))) return rc;
    launch_ex(gemm_tc_kernel<true>, dim3(grid), dim3(128), GEMM_SMEM, st, 1, tmA, tmB, p);
  } else {
    if ((rc = ensure_smem(gemm_tc_kernel<false>, GEMM_SMEM))) return rc;
    launch_ex(gemm_tc_kernel<false>, dim3(grid), dim3(128), GEMM_SMEM, st, 1, tmA, tmB, p);
  }
  return launch_status();
}


extern "C" int sa3_gptq_gemm(const void* A, const void* qw, const float* sz, void* C, int M, int N, int K,
                             long long lda, long long ldc, int group_size, const sa3_epilogue* epi, void* stream) {
  if (!A || !qw || !sz || !C || M <= 0 || N <= 0 || K <= 0) return SA3_ERR_ARG;
  if (group_size <= 0 || group_size % 64 || K % group_size || N % GEMM_BN) return SA3_ERR_UNSUPPORTED;
  if (!aligned16(A) || !aligned16(qw) || !aligned16(sz) || !aligned16(C) || (lda % 8) || lda < K) return SA3_ERR_ALIGN;
  sa3_epilogue e{};
  if (epi) e = *epi;
  if (e.kind < SA3_EPI_STORE || e.kind > SA3_EPI_QK_NORM) return SA3_ERR_ARG;
  if (e.c_f32 && e.c_f16) return SA3_ERR_ARG;
  if (e.c_f16 && (e.kind == SA3_EPI_SWIGLU || e.kind == SA3_EPI_QK_NORM)) return SA3_ERR_UNSUPPORTED;
  const int celt = e.c_f32 ? 4 : 2;
  if ((ldc * celt) % 16) return SA3_ERR_ALIGN;
  if (e.kind == SA3_EPI_SWIGLU ? ldc < N / 2 : ldc < N) return SA3_ERR_ARG;
  if (e.kind == SA3_EPI_SWIGLU && e.c_f32) return SA3_ERR_UNSUPPORTED;
  const bool res_kind = e.kind == SA3_EPI_GATED_RESIDUAL || e.kind == SA3_EPI_RESIDUAL;
  if (res_kind && (!e.residual || !aligned16(e.residual) || (e.ld_residual * celt) % 16)) return SA3_ERR_ARG;
  if (e.kind == SA3_EPI_GATED_RESIDUAL &&
      (!e.gate || !aligned16(e.gate) || e.ld_gate % 4 || (!e.row_batch && e.rows_per_batch <= 0)))
    return SA3_ERR_ARG;
  if (e.bias && !aligned16(e.bias)) return SA3_ERR_ALIGN;
  if (e.kind == SA3_EPI_QK_NORM) {
    if (e.qk_group_width <= 0 || e.qk_group_width % 64 || N > 8 * e.qk_group_width) return SA3_ERR_ARG;
    if (e.qk_rope_mask && (!e.cos_sin || e.max_pos <= 0 || (!e.row_pos && e.rows_per_batch <= 0)))
      return SA3_ERR_ARG;
  }
  if (e.seg_in < 0 || (e.seg_in > 0 && e.seg_out <= 0)) return SA3_ERR_ARG;
  CUtensorMap tmA, tmW, tmSZ;
  int rc;
  if ((rc = make_tmap_2d(&tmA, A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, M, lda, 64, GEMM_BM))) return rc;
  if ((rc = make_tmap_2d(&tmW, qw, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, K / 8, N, K / 8, 8, GEMM_BN,
                         CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  const int G = K / group_size;
  if ((rc = make_tmap_2d(&tmSZ, sz, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, 2 * (uint64_t)N, G, 2 * (uint64_t)N, 256, 1,
                         CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  GemmParams p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.ldc = ldc;
  p.C = C;
  p.a_scale = nullptr;
  p.b_scale = nullptr;
  p.epi = e;
  p.tma_store = 0;
  const int tiles_n = N / GEMM_BN;
  const int num_tiles = tiles_n * ((M + GEMM_BM - 1) / GEMM_BM);
  int sms = 0, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (sms <= 0) sms = 148;
  const int grid = num_tiles < sms ? num_tiles : sms;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
#define SA3_GQ_CASE(K_)                                                                                        \
  case K_:                                                                                                     \
    if ((rc = ensure_smem(gemm_gptq_kernel<K_>, GQ_SMEM))) return rc;                                          \
    launch_ex(gemm_gptq_kernel<K_>, dim3(grid), dim3(GQ_THREADS), GQ_SMEM, st, 1, tmA, tmW, tmSZ, p, tiles_n, num_tiles, group_size); \
    break;
  switch (e.kind) {
    SA3_GQ_CASE(SA3_EPI_STORE)
    SA3_GQ_CASE(SA3_EPI_SILU)
    SA3_GQ_CASE(SA3_EPI_SWIGLU)
    SA3_GQ_CASE(SA3_EPI_GATED_RESIDUAL)
    SA3_GQ_CASE(SA3_EPI_RESIDUAL)
    SA3_GQ_CASE(SA3_EPI_QK_NORM)
    default:
      return SA3_ERR_ARG;
  }
#undef SA3_GQ_CASE
  return launch_status();
}

extern "C" int sa3_gptq_dequant(const void* qw, const float* sz, void* out, int N, int K, int group_size,
                                void* stream) {
  if (!qw || !sz || !out || N <= 0 || K <= 0 || K % 8 || group_size <= 0 || K % group_size) return SA3_ERR_ARG;
  if (!aligned16(out) || K % 8) return SA3_ERR_ALIGN;
  const long long words = (long long)N * (K / 8);
  long long grid = (words + 255) / 256;
  if (grid > 148 * 16) grid = 148 * 16;
  launch_ex(gptq_dequant_kernel, dim3((int)grid), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), 1, 
      reinterpret_cast<const uint32_t*>(qw), sz, reinterpret_cast<__nv_bfloat16*>(out), N, K, group_size);
  return launch_status();
}

extern "C" int sa3_gptq_dequant_orig(const void* qw, const float* sz, const int* inv_perm, void* out, int N, int K,
                                     long long ldo, int group_size, void* stream) {
  if (!qw || !sz || !inv_perm || !out || N <= 0 || K <= 0 || K % 8 || group_size <= 0 || K % group_size ||
      ldo < K)
    return SA3_ERR_ARG;
  if (!aligned16(out) || !aligned16(inv_perm) || !aligned16(qw) || ldo % 8) return SA3_ERR_ALIGN;
  const int smem = K / 2 + (K / group_size) * 8;
  if (smem > 48 * 1024) return SA3_ERR_UNSUPPORTED;
  const int grid = N < 148 * 8 ? N : 148 * 8;
  launch_ex(gptq_dequant_orig_kernel, dim3(grid), dim3(256), smem, reinterpret_cast<cudaStream_t>(stream), 1,
            reinterpret_cast<const uint32_t*>(qw), sz, inv_perm, reinterpret_cast<__nv_bfloat16*>(out), N, K, ldo,
            group_size);
  return launch_status();
}

extern "C" int sa3_permute_cols(const void* x, const int* perm, void* out, int rows, int K, long long ldx,
                                long long ldo, void* stream) {
  if (!x || !perm || !out || rows <= 0 || K <= 0 || K % 8 || ldx < K || ldo < K) return SA3_ERR_ARG;
  if (!aligned16(x) || !aligned16(out) || !aligned16(perm) || ldx % 8 || ldo % 8) return SA3_ERR_ALIGN;
  const int smem = K * 2;
  if (smem > 96 * 1024) return SA3_ERR_UNSUPPORTED;
  int rc;
  // the attribute is set once per device, so set it to the largest row this kernel accepts
  if ((rc = ensure_smem(permute_cols_kernel, 96 * 1024))) return rc;
  const int grid = rows < 148 * 8 ? rows : 148 * 8;
  launch_ex(permute_cols_kernel, dim3(grid), dim3(256), smem, reinterpret_cast<cudaStream_t>(stream), 1, 
      reinterpret_cast<const __nv_bfloat16*>(x), perm, reinterpret_cast<__nv_bfloat16*>(out), rows, K, ldx, ldo);
  return launch_status();
}
