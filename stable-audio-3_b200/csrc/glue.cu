// Fused elementwise glue of the DiT block (HBM-bound; 128-bit vector access).
//
//   rmsnorm_modulate : RMSNorm (stable_audio_3/models/transformer.py:392-410)
//                      + adaLN modulate x*(1+scale)+shift (transformer.py:1018-1026,
//                      1043-1045), optionally writing e4m3 with the per-tensor
//                      dynamic activation scale, or only reducing max|y|.
//   quantize_e4m3    : per-tensor dynamic FP8 quantisation of a bf16 tensor.
//   qk_norm_rope     : per-head RMSNorm of q/k (Attention.apply_qk_layernorm,
//                      transformer.py:589-595) + partial rotary embedding on the
//                      first 32 of 64 dims, fp32 math (apply_rotary_pos_emb /
//                      rotate_half, transformer.py:296-322; use at :755-781).
#include <type_traits>

#include "common.cuh"
#include "host_util.h"

namespace sa3 {
SA3_DEFINE_ERROR_READER(read_error_glue)

constexpr float kE4M3Max = 448.f;

// Dynamic per-tensor FP8 scale: s = max(amax, 1e-12) / 448 dequantises; q = e4m3(x * inv) with
// inv = 448 / max(amax, 1e-12) quantises (one IEEE division per thread, a multiply per element).
__device__ __forceinline__ float quant_scale(const float* amax) { return fmaxf(__ldg(amax), 1e-12f) / kE4M3Max; }
__device__ __forceinline__ float quant_inv_scale(const float* amax) { return kE4M3Max / fmaxf(__ldg(amax), 1e-12f); }

__device__ __forceinline__ void unpack8_f16(const uint4& u, float (&v)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __half22float2(h[j]);
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}

__device__ __forceinline__ void unpack8(const uint4& u, float (&v)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 f = __bfloat1622float2(h[j]);
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}
__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  uint4 u;
  u.x = pack_bf16x2(v[0], v[1]);
  u.y = pack_bf16x2(v[2], v[3]);
  u.z = pack_bf16x2(v[4], v[5]);
  u.w = pack_bf16x2(v[6], v[7]);
  return u;
}
// q = e4m3(v * inv), saturating round-to-nearest-even (the oracle's definition).
// Two fp32 -> two e4m3 (round to nearest even, saturating to +-448) in one instruction; the
// first operand lands in the high byte, so (b, a) puts a in the lower byte.
__device__ __forceinline__ uint32_t e4m3x2(float a, float b) {
  uint16_t d;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(d) : "f"(b), "f"(a));
  return d;
}
__device__ __forceinline__ uint2 pack8_e4m3(const float (&v)[8], float inv) {
  const uint32_t lo = e4m3x2(v[0] * inv, v[1] * inv) | (e4m3x2(v[2] * inv, v[3] * inv) << 16);
  const uint32_t hi = e4m3x2(v[4] * inv, v[5] * inv) | (e4m3x2(v[6] * inv, v[7] * inv) << 16);
  return make_uint2(lo, hi);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-level max then one atomic per block.
__device__ __forceinline__ void block_amax_commit(float v, float* amax_out) {
  __shared__ float red[32];
  v = warp_max(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float w = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
    w = warp_max(w);
    if (lane == 0) atomic_max_nonneg(amax_out, w);
  }
}

struct NormParams {
  const void* x;
  int x_f32;
  int x_f16;  // the fp16 residual stream (x_f32 zero)
  void* out;
  int rows, D;
  long long ldx, ldo;
  const float* gamma;
  float eps;
  const float* mod;
  long long ld_mod;
  int scale_off, shift_off;
  int rows_per_batch;
  const int* row_batch;
  int mode, out_dtype;
  const float* quant_amax;
  float* scale_out;
  float* amax_out;
  float* row_r;  // optional [rows]: 1/rms of each row, stored by the AMAX pass, read by the WRITE pass
};

__device__ __forceinline__ void ld8f(const float* p, float (&v)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

template <int MAXC>
__device__ __forceinline__ void norm_load_row(const NormParams& p, int row, float (&v)[MAXC][8]) {
  const int lane = threadIdx.x & 31;
  const int nchunk = p.D / 8;
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = lane + i * 32;
    if (c < nchunk) {
      if (p.x_f32) {
        const float4* xr =
            reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.x) + (long long)row * p.ldx + c * 8);
        const float4 a = xr[0], b = xr[1];
        v[i][0] = a.x; v[i][1] = a.y; v[i][2] = a.z; v[i][3] = a.w;
        v[i][4] = b.x; v[i][5] = b.y; v[i][6] = b.z; v[i][7] = b.w;
      } else if (p.x_f16) {
        const __half* xr = reinterpret_cast<const __half*>(p.x) + (long long)row * p.ldx;
        unpack8_f16(*reinterpret_cast<const uint4*>(xr + c * 8), v[i]);
      } else {
        const __nv_bfloat16* xr = reinterpret_cast<const __nv_bfloat16*>(p.x) + (long long)row * p.ldx;
        unpack8(*reinterpret_cast<const uint4*>(xr + c * 8), v[i]);
      }
    }
  }
}

// Row visiting order. The fp32 stream was just written by a GEMM that walks its row tiles upwards,
// so the max|y| pass visits rows from the top down (the most recently written rows are still in
// L2), and the write pass that follows goes upwards again (the rows the max|y| pass read last).
__device__ __forceinline__ int norm_row(const NormParams& p, int i) {
  return p.mode == SA3_NORM_AMAX ? p.rows - 1 - i : i;
}

// One warp per row; each lane owns chunks of 8 columns at lane*8 + i*256. Warps are persistent and
// load row r + stride before normalising row r, so two rows of every warp are in flight. VEC: gamma
// and the modulation rows are 16-byte aligned and come in as float4 loads.
template <int MAXC, bool VEC>
__global__ void __launch_bounds__(128) rmsnorm_modulate_kernel(NormParams p) {
  grid_dep_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nchunk = p.D / 8;
  float s = 1.f;
  if (p.mode == SA3_NORM_WRITE && p.out_dtype == SA3_DT_E4M3) {
    s = quant_inv_scale(p.quant_amax);
    if (p.scale_out && blockIdx.x == 0 && threadIdx.x == 0) *p.scale_out = quant_scale(p.quant_amax);
  }
  float amax = 0.f;
  const int stride = gridDim.x * (blockDim.x >> 5);
  int li = blockIdx.x * (blockDim.x >> 5) + warp;
  float v[MAXC][8];
  if (li < p.rows) norm_load_row<MAXC>(p, norm_row(p, li), v);
  while (li < p.rows) {
    const int row = norm_row(p, li);
    const int nli = li + stride;
    float nv[MAXC][8];
    if (nli < p.rows) norm_load_row<MAXC>(p, norm_row(p, nli), nv);
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < MAXC; ++i)
      if (lane + i * 32 < nchunk) {
#pragma unroll
        for (int j = 0; j < 8; ++j) ss = fmaf(v[i][j], v[i][j], ss);
      }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / (float)p.D + p.eps);
    const float* msc = nullptr;
    const float* msh = nullptr;
    if (p.mod) {
      const int b = p.row_batch ? __ldg(p.row_batch + row) : row / p.rows_per_batch;
      msc = p.mod + (long long)b * p.ld_mod + p.scale_off;
      msh = p.mod + (long long)b * p.ld_mod + p.shift_off;
    }
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = lane + i * 32;
      if (c < nchunk) {
        float y[8], gm[8], sc[8], sh[8];
        if (VEC) {
          if (p.gamma) ld8f(p.gamma + c * 8, gm);
          if (msc) {
            ld8f(msc + c * 8, sc);
            ld8f(msh + c * 8, sh);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            gm[j] = p.gamma ? __ldg(p.gamma + c * 8 + j) : 1.f;
            sc[j] = msc ? __ldg(msc + c * 8 + j) : 0.f;
            sh[j] = msh ? __ldg(msh + c * 8 + j) : 0.f;
          }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float t = v[i][j] * r;
          if (p.gamma) t *= gm[j];
          if (msc) t = fmaf(t, 1.f + sc[j], sh[j]);
          y[j] = t;
        }
        if (p.mode == SA3_NORM_AMAX) {
#pragma unroll
          for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(y[j]));
        } else if (p.out_dtype == SA3_DT_E4M3) {
          uint8_t* o = reinterpret_cast<uint8_t*>(p.out) + (long long)row * p.ldo + c * 8;
          *reinterpret_cast<uint2*>(o) = pack8_e4m3(y, s);
        } else {
          __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.out) + (long long)row * p.ldo + c * 8;
          *reinterpret_cast<uint4*>(o) = pack8(y);
        }
      }
    }
    if (nli < p.rows) {
#pragma unroll
      for (int i = 0; i < MAXC; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = nv[i][j];
    }
    li = nli;
  }
  if (p.mode == SA3_NORM_AMAX) block_amax_commit(amax, p.amax_out);
}

// Direct-load variant for the fp32 stream: 8 warps per block, one row per warp at a time, lane l
// owning the float4s l + 32 k of the row, so every warp load is 512 contiguous bytes. The modulation
// coefficients a = gamma * (1 + scale) and shift of up to two CFG batches sit in a shared-memory table;
// rows of other batches (packed variable-length inputs) read them from global memory.
// Latency structure (a warp sees only ~7 rows at the medium shape, so nothing reaches a steady state
// unless loads are issued early): the first row of every warp is requested before the table is built,
// the table loads are all issued before any is used, and with DB the next row is loaded while the
// current one is normalised (2 rows per warp, 16 warps per SM in flight).
constexpr int NORM_D_THREADS = 256;
constexpr int NORM_D_TAB_IT = 4;  // table float4s per thread: tab_batches * D / 4 <= 4 * 256 (D <= 2048)

// L2 eviction policy of the row loads: the max|y| pass keeps the rows it reads (evict_last) for the
// write pass that follows, which reads them for the last time (evict_first).
__device__ __forceinline__ uint64_t norm_l2_policy(int mode) {
  uint64_t pol;
  if (mode == SA3_NORM_AMAX)
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  else
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ float4 ld_f4_hint(const float4* ptr, uint64_t pol) {
  float4 v;
  asm volatile("ld.global.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(ptr), "l"(pol));
  return v;
}
template <int NV>
__device__ __forceinline__ void norm_load_row4(const NormParams& p, int row, int lane, uint64_t pol, float4 (&v)[NV]) {
  const float4* xr = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.x) + (long long)row * p.ldx);
#pragma unroll
  for (int k = 0; k < NV; ++k) v[k] = ld_f4_hint(xr + lane + 32 * k, pol);
}
// fp16 stream: the same four elements per (lane, k) as the fp32 kernel, in one 8-byte load, kept packed until
// used so the loads stay in flight.
__device__ __forceinline__ uint2 ld_u2_hint(const uint2* ptr, uint64_t pol) {
  uint2 v;
  asm volatile("ld.global.L2::cache_hint.v2.u32 {%0, %1}, [%2], %3;" : "=r"(v.x), "=r"(v.y) : "l"(ptr), "l"(pol));
  return v;
}
template <int NV>
__device__ __forceinline__ void norm_load_row4(const NormParams& p, int row, int lane, uint64_t pol, uint2 (&v)[NV]) {
  const uint2* xr = reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(p.x) + (long long)row * p.ldx);
#pragma unroll
  for (int k = 0; k < NV; ++k) v[k] = ld_u2_hint(xr + lane + 32 * k, pol);
}
__device__ __forceinline__ float4 norm_f4(const float4& v) { return v; }
__device__ __forceinline__ float4 norm_f4(const uint2& v) {
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

// CFG batch of a row for the modulation table (every lane reads the same entry: one transaction).
__device__ __forceinline__ int norm_batch_load(const NormParams& p, int row) {
  if (!p.mod) return 0;
  if (!p.row_batch) return row / p.rows_per_batch;
  return __ldg(p.row_batch + row);
}

// NV groups of four elements per lane: D = 128 * NV; DB: next row prefetched; XH: the stream is fp16 (8-byte loads)
// Blocks per SM (register-limited at 128 per thread with a prefetched row). Three blocks of the fp16-stream variant at 80
// registers spill and ran slower (41.5 vs 38.0 us per norm pair at the medium shape).
template <int NV, bool DB, bool XH>
constexpr int norm_direct_blocks() { return (DB || NV > 12) ? 2 : 3; }

template <int NV, bool DB, bool XH>
__device__ __forceinline__ void norm_direct_body(const NormParams& p, int tab_batches, float* ntab) {
  using Raw = typename std::conditional<XH, uint2, float4>::type;  // the fp16 stream is kept packed until used
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = gridDim.x * (NORM_D_THREADS / 32);
  int li = blockIdx.x * (NORM_D_THREADS / 32) + warp;
  const uint64_t pol = norm_l2_policy(p.mode);
  Raw v[NV];
  int vb = 0;  // CFG batch of the row in v, requested with the row so its latency overlaps the row's
  if (li < p.rows) {
    vb = norm_batch_load(p, norm_row(p, li));
    norm_load_row4<NV>(p, norm_row(p, li), lane, pol, v);
  }
  {
    const int D4 = p.D >> 2, n4 = tab_batches * D4;
    float4 ta[NORM_D_TAB_IT], ts[NORM_D_TAB_IT];
#pragma unroll
    for (int it = 0; it < NORM_D_TAB_IT; ++it) {
      const int idx = threadIdx.x + it * NORM_D_THREADS;
      if (idx < n4) {
        const int b = idx / D4, e = 4 * (idx - b * D4);
        const float4 g = p.gamma ? __ldg(reinterpret_cast<const float4*>(p.gamma + e)) : make_float4(1.f, 1.f, 1.f, 1.f);
        if (p.mod) {
          const float4 sc = __ldg(reinterpret_cast<const float4*>(p.mod + (long long)b * p.ld_mod + p.scale_off + e));
          ts[it] = __ldg(reinterpret_cast<const float4*>(p.mod + (long long)b * p.ld_mod + p.shift_off + e));
          ta[it] = make_float4(g.x * (1.f + sc.x), g.y * (1.f + sc.y), g.z * (1.f + sc.z), g.w * (1.f + sc.w));
        } else {
          ta[it] = g;
          ts[it] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
    }
#pragma unroll
    for (int it = 0; it < NORM_D_TAB_IT; ++it) {
      const int idx = threadIdx.x + it * NORM_D_THREADS;
      if (idx < n4) {
        const int b = idx / D4, e = 4 * (idx - b * D4);
        *reinterpret_cast<float4*>(ntab + (2 * b) * p.D + e) = ta[it];
        *reinterpret_cast<float4*>(ntab + (2 * b + 1) * p.D + e) = ts[it];
      }
    }
  }
  __syncthreads();
  float s = 1.f;
  if (p.mode == SA3_NORM_WRITE && p.out_dtype == SA3_DT_E4M3) {
    s = quant_inv_scale(p.quant_amax);
    if (p.scale_out && blockIdx.x == 0 && threadIdx.x == 0) *p.scale_out = quant_scale(p.quant_amax);
  }
  float amax = 0.f;
  while (li < p.rows) {
    const int row = norm_row(p, li);
    const int nli = li + nw;
    Raw nv[DB ? NV : 1];
    int nvb = 0;
    if (DB && nli < p.rows) {
      nvb = norm_batch_load(p, norm_row(p, nli));
      norm_load_row4<DB ? NV : 1>(p, norm_row(p, nli), lane, pol, nv);
    }
    float ss4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const float4 x = norm_f4(v[k]);
      ss4[0] = fmaf(x.x, x.x, ss4[0]);
      ss4[1] = fmaf(x.y, x.y, ss4[1]);
      ss4[2] = fmaf(x.z, x.z, ss4[2]);
      ss4[3] = fmaf(x.w, x.w, ss4[3]);
    }
    const float r = rsqrtf(warp_sum((ss4[0] + ss4[1]) + (ss4[2] + ss4[3])) / (float)p.D + p.eps);
    if (p.mode == SA3_NORM_AMAX && p.row_r && lane == 0) p.row_r[row] = r;
    const int b = vb;
    const bool in_tab = b < tab_batches;  // warp-uniform
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int e = 4 * (lane + 32 * k);  // first element of this float4
      float4 a, sh;
      if (in_tab) {
        a = *reinterpret_cast<const float4*>(ntab + (2 * b) * p.D + e);
        sh = *reinterpret_cast<const float4*>(ntab + (2 * b + 1) * p.D + e);
      } else {
        const float4 g = p.gamma ? __ldg(reinterpret_cast<const float4*>(p.gamma + e)) : make_float4(1.f, 1.f, 1.f, 1.f);
        if (p.mod) {
          const float4 sc = __ldg(reinterpret_cast<const float4*>(p.mod + (long long)b * p.ld_mod + p.scale_off + e));
          sh = __ldg(reinterpret_cast<const float4*>(p.mod + (long long)b * p.ld_mod + p.shift_off + e));
          a = make_float4(g.x * (1.f + sc.x), g.y * (1.f + sc.y), g.z * (1.f + sc.z), g.w * (1.f + sc.w));
        } else {
          a = g;
          sh = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      const float4 x = norm_f4(v[k]);
      const float y0 = fmaf(x.x * r, a.x, sh.x), y1 = fmaf(x.y * r, a.y, sh.y);
      const float y2 = fmaf(x.z * r, a.z, sh.z), y3 = fmaf(x.w * r, a.w, sh.w);
      if (p.mode == SA3_NORM_AMAX) {
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(y0), fabsf(y1)), fmaxf(fabsf(y2), fabsf(y3))));
      } else if (p.out_dtype == SA3_DT_E4M3) {
        *reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(p.out) + (long long)row * p.ldo + e) =
            e4m3x2(y0 * s, y1 * s) | (e4m3x2(y2 * s, y3 * s) << 16);
      } else {
        *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p.out) + (long long)row * p.ldo + e) =
            make_uint2(pack_bf16x2(y0, y1), pack_bf16x2(y2, y3));
      }
    }
    if (DB) {
#pragma unroll
      for (int k = 0; k < NV; ++k) v[k] = nv[DB ? k : 0];
      vb = nvb;
    } else if (nli < p.rows) {
      vb = norm_batch_load(p, norm_row(p, nli));
      norm_load_row4<NV>(p, norm_row(p, nli), lane, pol, v);
    }
    li = nli;
  }
  if (p.mode == SA3_NORM_AMAX) block_amax_commit(amax, p.amax_out);
}

template <int NV, bool DB, bool XH>
__global__ void __launch_bounds__(NORM_D_THREADS, norm_direct_blocks<NV, DB, XH>()) rmsnorm_direct_kernel(NormParams p, int tab_batches) {
  grid_dep_wait();
  extern __shared__ __align__(16) float ntab[];  // [tab_batches][2][D]
  norm_direct_body<NV, DB, XH>(p, tab_batches, ntab);
}

// WRITE pass from the per-row 1/rms that the AMAX pass stored (p.row_r): no row reductions are left, so
// the pass is an elementwise stream over 8-element chunks with NORM_APPLY_INFLIGHT independent loads per
// thread (the structure of quantize_e4m3_kernel), y = fmaf(x * r, a, shift) with the modulation
// coefficients of the row's CFG batch from a shared-memory table: the same operations, in the same
// order, as the direct kernel's WRITE pass, so the output is identical. The first chunks' loads are
// issued before the table is built, so the table's loads overlap them. tab_batches (1 or 2) uniform
// batches of rows_per_batch rows. The fp16 stream only: on the fp32 stream this pass was no faster than
// the direct kernel's (24.0 vs 23.6 us at the medium shape). Coefficients from L1-cached global loads
// instead of the table: 25.7 us against 20.0 us.
constexpr int NORM_APPLY_INFLIGHT = 8;

struct NormApplyChunks {
  uint4 u[NORM_APPLY_INFLIGHT];  // 8 fp16 values each
  float rr[NORM_APPLY_INFLIGHT];
};

// (row, chunk) stepping by a fixed (dr, dc) per chunk, as in quantize_e4m3_kernel
__device__ __forceinline__ void norm_apply_step(int& r, int& c, int dr, int dc, int cpr) {
  r += dr;
  c += dc;
  if (c >= cpr) {
    c -= cpr;
    ++r;
  }
}

// FUSED: row_r was written earlier in the same launch by other blocks, so it is read through L2 (__ldcg), not
// through the read-only path.
template <bool FUSED>
__device__ __forceinline__ void norm_apply_load(const NormParams& p, NormApplyChunks& ch, int r, int c, int dr, int dc,
                                                int cpr) {
#pragma unroll
  for (int k = 0; k < NORM_APPLY_INFLIGHT; ++k) {
    if (r < p.rows) {
      ch.u[k] = *reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(p.x) + (long long)r * p.ldx + c * 8);
      ch.rr[k] = FUSED ? __ldcg(p.row_r + r) : __ldg(p.row_r + r);
    }
    norm_apply_step(r, c, dr, dc, cpr);
  }
}

// FUSED: the table in ntab was built by the max|y| pass of the same launch, and the scale is read through L2.
template <bool FUSED>
__device__ __forceinline__ void norm_apply_body(const NormParams& p, int tab_batches, float* ntab) {
  constexpr int NF = NORM_APPLY_INFLIGHT;
  const int cpr = p.D / 8;  // 8-element chunks per row
  const long long total = (long long)p.rows * cpr;
  const long long stride = (long long)gridDim.x * blockDim.x;
  const int dr = (int)(stride / cpr), dc = (int)(stride % cpr);
  long long i0 = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  int r0 = (int)(i0 / cpr), c0 = (int)(i0 % cpr);
  NormApplyChunks ch;
  norm_apply_load<FUSED>(p, ch, r0, c0, dr, dc, cpr);
  if (!FUSED) {
    const int D4 = p.D >> 2, n4 = tab_batches * D4;
    for (int idx = threadIdx.x; idx < n4; idx += blockDim.x) {
      const int b = idx / D4, e = 4 * (idx - b * D4);
      const float4 g = p.gamma ? __ldg(reinterpret_cast<const float4*>(p.gamma + e)) : make_float4(1.f, 1.f, 1.f, 1.f);
      float4 ta, ts;
      if (p.mod) {
        const float4 sc = __ldg(reinterpret_cast<const float4*>(p.mod + (long long)b * p.ld_mod + p.scale_off + e));
        ts = __ldg(reinterpret_cast<const float4*>(p.mod + (long long)b * p.ld_mod + p.shift_off + e));
        ta = make_float4(g.x * (1.f + sc.x), g.y * (1.f + sc.y), g.z * (1.f + sc.z), g.w * (1.f + sc.w));
      } else {
        ta = g;
        ts = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      *reinterpret_cast<float4*>(ntab + (2 * b) * p.D + e) = ta;
      *reinterpret_cast<float4*>(ntab + (2 * b + 1) * p.D + e) = ts;
    }
  }
  if (!FUSED) __syncthreads();
  float s = 1.f;
  if (p.out_dtype == SA3_DT_E4M3) {
    if (FUSED) {
      const float am = fmaxf(__ldcg(p.quant_amax), 1e-12f);  // quant_inv_scale / quant_scale on the L2 value
      s = kE4M3Max / am;
      if (p.scale_out && blockIdx.x == 0 && threadIdx.x == 0) *p.scale_out = am / kE4M3Max;
    } else {
      s = quant_inv_scale(p.quant_amax);
      if (p.scale_out && blockIdx.x == 0 && threadIdx.x == 0) *p.scale_out = quant_scale(p.quant_amax);
    }
  }
  while (i0 < total) {
    int r = r0, c = c0;
#pragma unroll
    for (int k = 0; k < NF; ++k) {
      if (r < p.rows) {
        float x[8];
        const __half2* h = reinterpret_cast<const __half2*>(&ch.u[k]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __half22float2(h[j]);
          x[2 * j] = f.x;
          x[2 * j + 1] = f.y;
        }
        const int b = tab_batches == 2 && r >= p.rows_per_batch ? 1 : 0;
        const float4* ap = reinterpret_cast<const float4*>(ntab + (2 * b) * p.D + c * 8);
        const float4* sp = reinterpret_cast<const float4*>(ntab + (2 * b + 1) * p.D + c * 8);
        const float4 a0 = ap[0], a1 = ap[1], s0 = sp[0], s1 = sp[1];
        const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const float sh[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
        float y[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) y[j] = fmaf(x[j] * ch.rr[k], a[j], sh[j]);
        if (p.out_dtype == SA3_DT_E4M3) {
          *reinterpret_cast<uint2*>(reinterpret_cast<uint8_t*>(p.out) + (long long)r * p.ldo + c * 8) =
              make_uint2(e4m3x2(y[0] * s, y[1] * s) | (e4m3x2(y[2] * s, y[3] * s) << 16),
                         e4m3x2(y[4] * s, y[5] * s) | (e4m3x2(y[6] * s, y[7] * s) << 16));
        } else {
          *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.out) + (long long)r * p.ldo + c * 8) =
              make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]), pack_bf16x2(y[4], y[5]),
                         pack_bf16x2(y[6], y[7]));
        }
      }
      norm_apply_step(r, c, dr, dc, cpr);
    }
    r0 = r;
    c0 = c;
    i0 += NF * stride;
    if (i0 < total) norm_apply_load<FUSED>(p, ch, r0, c0, dr, dc, cpr);
  }
}

__global__ void __launch_bounds__(256, 3) norm_apply_kernel(NormParams p, int tab_batches) {
  grid_dep_wait();
  extern __shared__ __align__(16) float ntab[];  // [tab_batches][2][D]
  norm_apply_body<false>(p, tab_batches, ntab);
}

// Grid-wide barrier with sense reversal: bar[0] counts arrivals, bar[1] is the generation. A block reads the
// generation, then arrives; the last block to arrive resets the count and advances the generation, the others
// wait (bounded by SA3_WAIT_BUDGET_CYCLES, then device error site 95) for it to change. Every block of the grid
// must be resident at once (the host caps the grid at the kernel's occupancy).
__device__ __forceinline__ void norm_grid_barrier(unsigned int* bar) {
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned int gen;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(gen) : "l"(bar + 1) : "memory");
    __threadfence();
    if (atomicAdd(bar, 1u) == gridDim.x - 1) {
      bar[0] = 0u;
      __threadfence();
      atomicAdd(bar + 1, 1u);
    } else {
      const long long t0 = clock64();
      while (true) {
        unsigned int g;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(g) : "l"(bar + 1) : "memory");
        if (g != gen) break;
        if (clock64() - t0 > SA3_WAIT_BUDGET_CYCLES) {
          record_error(SA3_DEVERR_TIMEOUT, 95);
          break;
        }
        __nanosleep(64);
      }
    }
    __threadfence();
  }
  __syncthreads();
}

// One launch per norm of the fp16 stream: the max|y| pass (direct kernel body: 1/rms of every row into row_r,
// max|y| into amax_out), a grid barrier, then the elementwise e4m3 / bf16 write pass from row_r with the scale of
// the now complete max. Same operations as the two launches, so the same bytes.
template <int NV>
__global__ void __launch_bounds__(NORM_D_THREADS, 2) norm_fused_kernel(NormParams p, int tab_batches, unsigned int* bar) {
  grid_dep_wait();
  extern __shared__ __align__(16) float ntab[];  // [tab_batches][2][D]
  NormParams pa = p;
  pa.mode = SA3_NORM_AMAX;
  norm_direct_body<NV, true, true>(pa, tab_batches, ntab);
  norm_grid_barrier(bar);
  NormParams pw = p;
  pw.mode = SA3_NORM_WRITE;
  norm_apply_body<true>(pw, tab_batches, ntab);
}

// Bulk-copy variant: warp 4 (lane 0) streams whole rows into an NORM_RING-deep shared-memory ring
// with cp.async.bulk (one mbarrier per slot); warps 0..3 each normalise one row at a time from
// shared memory. Up to NORM_RING rows per block are in flight independently of the consumers.
constexpr int NORM_RING = 12;
constexpr int NORM_BULK_THREADS = 160;

template <int MAXC, bool VEC>
__global__ void __launch_bounds__(NORM_BULK_THREADS, 2) rmsnorm_bulk_kernel(NormParams p, int rowbytes) {
  grid_dep_wait();
  extern __shared__ __align__(16) uint8_t nsm[];
  uint64_t* full = reinterpret_cast<uint64_t*>(nsm + NORM_RING * rowbytes);
  uint64_t* empty = full + NORM_RING;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + NORM_RING);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nchunk = p.D / 8;
  // rows of this block: blockIdx.x + i * gridDim.x
  const int nrows = p.rows > (int)blockIdx.x ? (p.rows - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  if (threadIdx.x == 0) {
    for (int i = 0; i < NORM_RING; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  float s = 1.f;
  if (p.mode == SA3_NORM_WRITE && p.out_dtype == SA3_DT_E4M3) {
    s = quant_inv_scale(p.quant_amax);
    if (p.scale_out && blockIdx.x == 0 && threadIdx.x == 0) *p.scale_out = quant_scale(p.quant_amax);
  }
  float amax = 0.f;
  if (warp == 4) {
    if (lane == 0) {
      int li = 0;
      for (; li < nrows; ++li) {
        const int slot = li % NORM_RING;
        if (li >= NORM_RING && !mbar_wait(&empty[slot], ((li / NORM_RING) - 1) & 1, abort_flag, 60)) break;
        const int row = norm_row(p, blockIdx.x + li * gridDim.x);
        const uint8_t* src = reinterpret_cast<const uint8_t*>(p.x) + (long long)row * p.ldx * (p.x_f32 ? 4 : 2);
        mbar_arrive_expect_tx(&full[slot], rowbytes);
        bulk_load(nsm + slot * rowbytes, src, rowbytes, &full[slot]);
      }
      if (*abort_flag) {
        volatile int never = 0;
        for (int j = (li > NORM_RING ? li - NORM_RING : 0); j < li; ++j)
          mbar_wait(&full[j % NORM_RING], (j / NORM_RING) & 1, &never, 61);
      }
    }
  } else {
    int cur_b = -1;  // CFG batch whose coefficients ca hold (VEC)
    float ca[MAXC][8];
    for (int li = warp; li < nrows; li += 4) {
      const int slot = li % NORM_RING;
      if (!mbar_wait(&full[slot], (li / NORM_RING) & 1, abort_flag, 62)) break;
      const int row = norm_row(p, blockIdx.x + li * gridDim.x);
      const uint8_t* rb = nsm + slot * rowbytes;
      float v[MAXC][8];
      float ss4[4] = {0.f, 0.f, 0.f, 0.f};  // independent chains
#pragma unroll
      for (int i = 0; i < MAXC; ++i) {
        const int c = lane + i * 32;
        if (c < nchunk) {
          if (p.x_f32) {
            const float4 a = reinterpret_cast<const float4*>(rb)[2 * c];
            const float4 b = reinterpret_cast<const float4*>(rb)[2 * c + 1];
            v[i][0] = a.x; v[i][1] = a.y; v[i][2] = a.z; v[i][3] = a.w;
            v[i][4] = b.x; v[i][5] = b.y; v[i][6] = b.z; v[i][7] = b.w;
          } else if (p.x_f16) {
            unpack8_f16(reinterpret_cast<const uint4*>(rb)[c], v[i]);
          } else {
            unpack8(reinterpret_cast<const uint4*>(rb)[c], v[i]);
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) ss4[j & 3] = fmaf(v[i][j], v[i][j], ss4[j & 3]);
        }
      }
      float ss = (ss4[0] + ss4[1]) + (ss4[2] + ss4[3]);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);  // the row is in registers: the slot may refill
      ss = warp_sum(ss);
      const float r = rsqrtf(ss / (float)p.D + p.eps);
      const int b = p.mod ? (p.row_batch ? __ldg(p.row_batch + row) : row / p.rows_per_batch) : 0;
      if (VEC && b != cur_b) {
        // warp-uniform (one row per warp): y = x * r * a + shift with a = gamma * (1 + scale) held in
        // registers across rows of the same CFG batch; the shift row is read per row
        cur_b = b;
        const float* msc = p.mod ? p.mod + (long long)b * p.ld_mod + p.scale_off : nullptr;
#pragma unroll
        for (int i = 0; i < MAXC; ++i) {
          const int c = lane + i * 32;
          if (c < nchunk) {
            float gm[8], sc[8];
            if (p.gamma) ld8f(p.gamma + c * 8, gm);
            if (msc) ld8f(msc + c * 8, sc);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float g = p.gamma ? gm[j] : 1.f;
              ca[i][j] = msc ? g * (1.f + sc[j]) : g;
            }
          }
        }
      }
#pragma unroll
      for (int i = 0; i < MAXC; ++i) {
        const int c = lane + i * 32;
        if (c < nchunk) {
          float y[8];
          if (VEC) {
            float sh[8];
            if (p.mod) {
              ld8f(p.mod + (long long)b * p.ld_mod + p.shift_off + c * 8, sh);
            } else {
#pragma unroll
              for (int j = 0; j < 8; ++j) sh[j] = 0.f;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) y[j] = fmaf(v[i][j] * r, ca[i][j], sh[j]);
          } else {
            const float* msc = p.mod ? p.mod + (long long)b * p.ld_mod + p.scale_off : nullptr;
            const float* msh = p.mod ? p.mod + (long long)b * p.ld_mod + p.shift_off : nullptr;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              float t = v[i][j] * r;
              if (p.gamma) t *= __ldg(p.gamma + c * 8 + j);
              if (msc) t = fmaf(t, 1.f + __ldg(msc + c * 8 + j), __ldg(msh + c * 8 + j));
              y[j] = t;
            }
          }
          if (p.mode == SA3_NORM_AMAX) {
#pragma unroll
            for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(y[j]));
          } else if (p.out_dtype == SA3_DT_E4M3) {
            uint8_t* o = reinterpret_cast<uint8_t*>(p.out) + (long long)row * p.ldo + c * 8;
            *reinterpret_cast<uint2*>(o) = pack8_e4m3(y, s);
          } else {
            __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.out) + (long long)row * p.ldo + c * 8;
            *reinterpret_cast<uint4*>(o) = pack8(y);
          }
        }
      }
    }
  }
  if (p.mode == SA3_NORM_AMAX) {
    amax = warp_max(amax);
    if (lane == 0 && warp < 4) atomic_max_nonneg(p.amax_out, amax);
  }
}

struct QuantParams {
  const __nv_bfloat16* x;
  uint8_t* out;
  int rows, cols;
  long long ldx, ldo;
  const float* amax;
  float* scale_out;
  float* amax_out;
};

// Eight independent 16-byte loads per thread and three 256-thread blocks per SM keep ~96 KB per SM
// in flight, which the HBM latency needs. A thread walks its chunks with a fixed stride, so its
// (row, chunk) position advances by a precomputed (row, chunk) step instead of a division.
constexpr int QUANT_INFLIGHT = 8;
__global__ void __launch_bounds__(256, 3) quantize_e4m3_kernel(QuantParams p) {
  grid_dep_wait();
  const int cpr = p.cols / 8;  // 8-element chunks per row
  const long long total = (long long)p.rows * cpr;
  float s = 1.f;
  if (!p.amax_out) {
    s = quant_inv_scale(p.amax);
    if (p.scale_out && blockIdx.x == 0 && threadIdx.x == 0) *p.scale_out = quant_scale(p.amax);
  }
  float amax = 0.f;
  const long long stride = (long long)gridDim.x * blockDim.x;
  const int dr = (int)(stride / cpr), dc = (int)(stride % cpr);
  long long i0 = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  int r0 = (int)(i0 / cpr), c0 = (int)(i0 % cpr);
  for (; i0 < total; i0 += QUANT_INFLIGHT * stride) {
    uint4 u[QUANT_INFLIGHT];
    int r = r0, c = c0;
#pragma unroll
    for (int k = 0; k < QUANT_INFLIGHT; ++k) {
      if (r < p.rows) u[k] = *reinterpret_cast<const uint4*>(p.x + (long long)r * p.ldx + c * 8);
      r += dr;
      c += dc;
      if (c >= cpr) {
        c -= cpr;
        ++r;
      }
    }
    r = r0;
    c = c0;
#pragma unroll
    for (int k = 0; k < QUANT_INFLIGHT; ++k) {
      if (r < p.rows) {
        float v[8];
        unpack8(u[k], v);
        if (p.amax_out) {
#pragma unroll
          for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[j]));
        } else {
          *reinterpret_cast<uint2*>(p.out + (long long)r * p.ldo + c * 8) = pack8_e4m3(v, s);
        }
      }
      r += dr;
      c += dc;
      if (c >= cpr) {
        c -= cpr;
        ++r;
      }
    }
    r0 = r;
    c0 = c;
  }
  if (p.amax_out) block_amax_commit(amax, p.amax_out);
}

struct QkParams {
  __nv_bfloat16* buf;
  int rows;
  long long ld;
  int heads, ngroups;
  int col_off[4];
  const float* gamma[4];
  int rope[4];
  float eps;
  const float* cos_sin;
  int max_pos;
  int rows_per_batch;
  const int* row_pos;
};

// Eight lanes per 64-wide head, 8 elements per lane; a warp handles 4 heads.
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(QkParams p) {
  grid_dep_wait();
  const int lane = threadIdx.x & 31;
  const int sub = lane & 7;
  const int per_row = p.ngroups * p.heads;
  const long long total = (long long)p.rows * per_row;
  const long long warps_total = (long long)gridDim.x * (blockDim.x >> 5);
  const long long gw = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  for (long long base = gw * 4; base < total; base += warps_total * 4) {
    const long long item = base + (lane >> 3);
    const bool active = item < total;
    const long long row = active ? item / per_row : 0;
    const int gh = active ? (int)(item - row * per_row) : 0;
    const int g = gh / p.heads;
    const int h = gh - g * p.heads;
    // per-group parameters selected without indexing the parameter arrays (keeps them in registers)
    const int coff = g == 0 ? p.col_off[0] : g == 1 ? p.col_off[1] : g == 2 ? p.col_off[2] : p.col_off[3];
    const float* gm = g == 0 ? p.gamma[0] : g == 1 ? p.gamma[1] : g == 2 ? p.gamma[2] : p.gamma[3];
    const int rope = g == 0 ? p.rope[0] : g == 1 ? p.rope[1] : g == 2 ? p.rope[2] : p.rope[3];
    __nv_bfloat16* ptr = p.buf + row * p.ld + coff + h * 64 + sub * 8;
    float v[8];
    if (active) unpack8(*reinterpret_cast<const uint4*>(ptr), v);
    else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = 0.f;
    }
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(v[j], v[j], ss);
    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
    ss += __shfl_xor_sync(0xffffffffu, ss, 2);
    ss += __shfl_xor_sync(0xffffffffu, ss, 4);
    const float r = rsqrtf(ss * (1.f / 64.f) + p.eps);
    if (gm) {
      float gv[8];
      ld8f(gm + sub * 8, gv);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = v[j] * r * gv[j];
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] *= r;
    }
    // rotate_half pairs dim d with d +- 16: lanes sub and sub^2 within the first 32 dims.
    float partner[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) partner[j] = __shfl_xor_sync(0xffffffffu, v[j], 2);
    if (active && rope && sub < 4) {
      int pos = p.row_pos ? __ldg(p.row_pos + row) : (int)(row % p.rows_per_batch);
      if (pos >= p.max_pos) {
        record_error(2, 10);
        pos = p.max_pos - 1;
      }
      // dims sub*8 .. sub*8+7 use frequencies (sub & 1) * 8 .. +7
      const float* cs = p.cos_sin + (long long)pos * 32 + (sub & 1) * 8;
      float cv[8], sv[8];
      ld8f(cs, cv);
      ld8f(cs + 16, sv);
      const float sgn = sub < 2 ? -1.f : 1.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = fmaf(v[j], cv[j], sgn * partner[j] * sv[j]);
    }
    if (active) *reinterpret_cast<uint4*>(ptr) = pack8(v);
  }
}

struct ConvParams {
  const void* x;
  void* out;
  const int* src_rows;
  int x_dt, out_dt;  // SA3_DT_BF16 / SA3_DT_F16 / SA3_DT_F32
  int rows, cols;
  long long ldx, ldo;
};

__global__ void __launch_bounds__(256) convert_kernel(ConvParams p) {
  grid_dep_wait();
  const int cpr = p.cols / 8;
  const long long total = (long long)p.rows * cpr;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / cpr;
    const int c = (int)(i - r * cpr);
    const long long rs = p.src_rows ? (long long)__ldg(p.src_rows + r) : r;
    float v[8];
    if (p.x_dt == SA3_DT_F32) {
      const float4* s = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.x) + rs * p.ldx + c * 8);
      const float4 a = s[0], b = s[1];
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else if (p.x_dt == SA3_DT_F16) {
      const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(p.x) + rs * p.ldx + c * 8);
      const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(h[j]);
        v[2 * j] = f.x;
        v[2 * j + 1] = f.y;
      }
    } else {
      unpack8(*reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p.x) + rs * p.ldx + c * 8), v);
    }
    if (p.out_dt == SA3_DT_F32) {
      float4* d = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + r * p.ldo + c * 8);
      d[0] = make_float4(v[0], v[1], v[2], v[3]);
      d[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else if (p.out_dt == SA3_DT_F16) {
      uint4 u;
      __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) h[j] = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
      *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(p.out) + r * p.ldo + c * 8) = u;
    } else {
      *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.out) + r * p.ldo + c * 8) = pack8(v);
    }
  }
}

inline int grid_for(long long work_items, int per_block) {
  long long g = (work_items + per_block - 1) / per_block;
  const long long cap = 148LL * 16;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (int)g;
}

}  // namespace sa3

using namespace sa3;

extern "C" int sa3_rmsnorm_modulate(const void* x, int x_dtype, void* out, int rows, int D, long long ldx,
                                    long long ldo, const float* gamma, float eps, const float* mod, long long ld_mod, int scale_off,
                                    int shift_off, int rows_per_batch, const int* row_batch, int mode, int out_dtype,
                                    const float* quant_amax, float* scale_out, float* amax_out, float* row_r,
                                    void* stream) {
  if (!x || rows <= 0 || D <= 0 || (D % 8) || ldx < D) return SA3_ERR_ARG;
  if (x_dtype != SA3_DT_BF16 && x_dtype != SA3_DT_F32 && x_dtype != SA3_DT_F16) return SA3_ERR_DTYPE;
  if (!aligned16(x) || (ldx % 8)) return SA3_ERR_ALIGN;
  if (mode == SA3_NORM_AMAX) {
    if (!amax_out) return SA3_ERR_ARG;
  } else if (mode == SA3_NORM_WRITE) {
    if (!out || ldo < D) return SA3_ERR_ARG;
    if (out_dtype == SA3_DT_E4M3) {
      if (!quant_amax) return SA3_ERR_ARG;
      if ((reinterpret_cast<uintptr_t>(out) & 7) || (ldo % 8)) return SA3_ERR_ALIGN;
    } else if (out_dtype == SA3_DT_BF16) {
      if (!aligned16(out) || (ldo % 8)) return SA3_ERR_ALIGN;
    } else {
      return SA3_ERR_DTYPE;
    }
  } else {
    return SA3_ERR_ARG;
  }
  if (mod && !row_batch && rows_per_batch <= 0) return SA3_ERR_ARG;
  NormParams p;
  p.x = x;
  p.x_f32 = x_dtype == SA3_DT_F32;
  p.x_f16 = x_dtype == SA3_DT_F16;
  p.out = out;
  p.rows = rows;
  p.D = D;
  p.ldx = ldx;
  p.ldo = ldo;
  p.gamma = gamma;
  p.eps = eps;
  p.mod = mod;
  p.ld_mod = ld_mod;
  p.scale_off = scale_off;
  p.shift_off = shift_off;
  p.rows_per_batch = rows_per_batch;
  p.row_batch = row_batch;
  p.mode = mode;
  p.out_dtype = out_dtype;
  p.quant_amax = quant_amax;
  p.scale_out = scale_out;
  p.amax_out = amax_out;
  p.row_r = nullptr;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int nchunk = D / 8;
  int grid = (rows + 3) / 4;  // 4 warps (rows) per 128-thread block
  if (grid > 148 * 3) grid = 148 * 3;  // one wave at 3 blocks per SM
  const bool vec = aligned16(gamma) && (!mod || (aligned16(mod) && ld_mod % 4 == 0 && scale_off % 4 == 0 &&
                                                    shift_off % 4 == 0));
  const int rowbytes = D * (x_dtype == SA3_DT_F32 ? 4 : 2);
  const bool xh = x_dtype == SA3_DT_F16;
  if (vec && (x_dtype == SA3_DT_F32 || xh) && D % 128 == 0 && D <= 4096 && ldx % 4 == 0 &&
      (mode == SA3_NORM_AMAX || out_dtype == SA3_DT_BF16 ? (ldo % 4 == 0) : (ldo % 4 == 0))) {
    int tab_batches = 1;
    if (mod) tab_batches = (!row_batch && rows_per_batch > 0 && (rows + rows_per_batch - 1) / rows_per_batch <= 2)
                               ? (rows + rows_per_batch - 1) / rows_per_batch
                               : 0;
    const int smem = tab_batches * 2 * D * 4;
    int gridd = (rows + 7) / 8;
    int rc;
    // row_r is stored and used only where the direct kernel runs both passes (D / 128 = 8, 12 or 16)
    const bool direct = D / 128 == 8 || D / 128 == 12 || D / 128 == 16;
    if (row_r && direct && mode == SA3_NORM_AMAX) p.row_r = row_r;  // the direct kernel stores 1/rms per row
    if (row_r && direct && xh && mode == SA3_NORM_WRITE && (tab_batches >= 1 || !mod) && aligned16(x) &&
        ldx % 8 == 0 && (out_dtype == SA3_DT_E4M3 || aligned16(out))) {
      // 1/rms of every row is known: the WRITE pass is an elementwise stream
      p.row_r = row_r;
      const int tb = mod ? tab_batches : 1;
      const long long chunks = (long long)rows * (D / 8);
      const long long per_block = 256LL * NORM_APPLY_INFLIGHT;
      long long ga = (chunks + per_block - 1) / per_block;
      if (ga > 148 * 3) ga = 148 * 3;
      const int smem_a = tb * 2 * D * 4;
      if ((rc = ensure_smem(norm_apply_kernel, 2 * 2 * 4096 * 4))) return rc;
      launch_ex(norm_apply_kernel, dim3((int)ga), dim3(256), smem_a, st, 1, p, tb);
      return launch_status();
    }
#define SA3_NORM_DIRECT(V, DB)                                                                                 \
  case V:                                                                                                      \
    if (xh) {                                                                                                  \
      if (gridd > 148 * norm_direct_blocks<V, DB, true>()) gridd = 148 * norm_direct_blocks<V, DB, true>();    \
      if ((rc = ensure_smem(rmsnorm_direct_kernel<V, DB, true>, 2 * 2 * 2048 * 4))) return rc;                 \
      launch_ex(rmsnorm_direct_kernel<V, DB, true>, dim3(gridd), dim3(NORM_D_THREADS), smem, st, 1, p, tab_batches); \
    } else {                                                                                                   \
      if (gridd > 148 * norm_direct_blocks<V, DB, false>()) gridd = 148 * norm_direct_blocks<V, DB, false>();  \
      if ((rc = ensure_smem(rmsnorm_direct_kernel<V, DB, false>, 2 * 2 * 2048 * 4))) return rc;                \
      launch_ex(rmsnorm_direct_kernel<V, DB, false>, dim3(gridd), dim3(NORM_D_THREADS), smem, st, 1, p, tab_batches); \
    }                                                                                                          \
    break;
    switch (D / 128) {
      SA3_NORM_DIRECT(8, true)
      SA3_NORM_DIRECT(12, true)
      SA3_NORM_DIRECT(16, false)
      default:
        goto bulk_path;
    }
#undef SA3_NORM_DIRECT
    return launch_status();
  }
bulk_path:
  if (rowbytes % 16 == 0 && rowbytes * NORM_RING <= 96 * 1024 && nchunk <= 32 * 8) {
    // bulk-copy pipeline: one row per slot; 2 blocks of 5 warps per SM (the consumers hold a row and
    // its modulation coefficients in registers), 2 x NORM_RING rows in flight per SM
    const int smem = NORM_RING * rowbytes + 2 * NORM_RING * 8 + 16;
    int gridb = rows < 148 * 2 ? rows : 148 * 2;
#define SA3_NORM_BULK(C)                                                                             \
  if (vec) {                                                                                         \
    if ((rc = ensure_smem(rmsnorm_bulk_kernel<C, true>, 96 * 1024 + 256))) return rc;                \
    launch_ex(rmsnorm_bulk_kernel<C, true>, dim3(gridb), dim3(NORM_BULK_THREADS), smem, st, 1, p, rowbytes);               \
  } else {                                                                                           \
    if ((rc = ensure_smem(rmsnorm_bulk_kernel<C, false>, 96 * 1024 + 256))) return rc;               \
    launch_ex(rmsnorm_bulk_kernel<C, false>, dim3(gridb), dim3(NORM_BULK_THREADS), smem, st, 1, p, rowbytes);              \
  }
    int rc;
    if (nchunk <= 32 * 4) {
      SA3_NORM_BULK(4)
    } else if (nchunk <= 32 * 6) {
      SA3_NORM_BULK(6)
    } else {
      SA3_NORM_BULK(8)
    }
#undef SA3_NORM_BULK
    return launch_status();
  }
#define SA3_NORM_LAUNCH(C)                                      \
  if (vec)                                                      \
    launch_ex(rmsnorm_modulate_kernel<C, true>, dim3(grid), dim3(128), 0, st, 1, p);  \
  else                                                          \
    launch_ex(rmsnorm_modulate_kernel<C, false>, dim3(grid), dim3(128), 0, st, 1, p);
  if (nchunk <= 32 * 4) {
    SA3_NORM_LAUNCH(4)
  } else if (nchunk <= 32 * 6) {
    SA3_NORM_LAUNCH(6)
  } else if (nchunk <= 32 * 8) {
    SA3_NORM_LAUNCH(8)
  } else if (nchunk <= 32 * 16) {
    SA3_NORM_LAUNCH(16)
  } else {
    return SA3_ERR_UNSUPPORTED;
  }
#undef SA3_NORM_LAUNCH
  return launch_status();
}

extern "C" int sa3_quantize_e4m3(const void* x, void* out, int rows, int cols, long long ldx, long long ldo,
                                 const float* amax, float* scale_out, float* amax_out, void* stream) {
  if (!x || rows <= 0 || cols <= 0 || (cols % 8) || ldx < cols) return SA3_ERR_ARG;
  if (!aligned16(x) || (ldx % 8)) return SA3_ERR_ALIGN;
  if (!amax_out) {
    if (!out || !amax || ldo < cols) return SA3_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(out) & 7) || (ldo % 8)) return SA3_ERR_ALIGN;
  }
  QuantParams p{reinterpret_cast<const __nv_bfloat16*>(x), reinterpret_cast<uint8_t*>(out), rows, cols, ldx, ldo,
                amax, scale_out, amax_out};
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  long long qgrid = ((long long)rows * (cols / 8) + 1023) / 1024;
  if (qgrid > 148 * 3) qgrid = 148 * 3;
  if (qgrid < 1) qgrid = 1;
  launch_ex(quantize_e4m3_kernel, dim3((int)qgrid), dim3(256), 0, st, 1, p);
  return launch_status();
}

extern "C" int sa3_qk_norm_rope(void* buf, int rows, long long ld, int heads, int ngroups, const int* col_off,
                                const float* const* gamma, const int* rope, float eps, const float* cos_sin,
                                int max_pos, int rows_per_batch, const int* row_pos, void* stream) {
  if (!buf || rows <= 0 || heads <= 0 || ngroups < 1 || ngroups > 4 || !col_off) return SA3_ERR_ARG;
  if (!aligned16(buf) || (ld % 8)) return SA3_ERR_ALIGN;
  QkParams p{};
  p.buf = reinterpret_cast<__nv_bfloat16*>(buf);
  p.rows = rows;
  p.ld = ld;
  p.heads = heads;
  p.ngroups = ngroups;
  bool any_rope = false;
  for (int g = 0; g < ngroups; ++g) {
    if (col_off[g] < 0 || (col_off[g] % 8) || col_off[g] + heads * 64 > ld) return SA3_ERR_ARG;
    p.col_off[g] = col_off[g];
    p.gamma[g] = gamma ? gamma[g] : nullptr;
    if (p.gamma[g] && !aligned16(p.gamma[g])) return SA3_ERR_ALIGN;
    p.rope[g] = rope ? rope[g] : 0;
    any_rope |= p.rope[g] != 0;
  }
  if (any_rope && (!cos_sin || max_pos <= 0 || (!row_pos && rows_per_batch <= 0))) return SA3_ERR_ARG;
  p.eps = eps;
  p.cos_sin = cos_sin;
  p.max_pos = max_pos;
  p.rows_per_batch = rows_per_batch;
  p.row_pos = row_pos;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const long long items = (long long)rows * ngroups * heads;
  launch_ex(qk_norm_rope_kernel, dim3(grid_for(items, 32)), dim3(256), 0, st, 1, p);
  return launch_status();
}

extern "C" int sa3_convert(const void* x, int x_dtype, void* out, int out_dtype, int rows, int cols, long long ldx,
                           long long ldo, const int* src_rows, void* stream) {
  if (!x || !out || rows <= 0 || cols <= 0 || (cols % 8) || ldx < cols || ldo < cols) return SA3_ERR_ARG;
  auto known = [](int d) { return d == SA3_DT_BF16 || d == SA3_DT_F16 || d == SA3_DT_F32; };
  if (!known(x_dtype) || !known(out_dtype)) return SA3_ERR_DTYPE;
  if (!aligned16(x) || !aligned16(out) || (ldx % 8) || (ldo % 8)) return SA3_ERR_ALIGN;
  ConvParams p{x, out, src_rows, x_dtype, out_dtype, rows, cols, ldx, ldo};
  launch_ex(convert_kernel, dim3(grid_for((long long)rows * (cols / 8), 256)), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), 1, p);
  return launch_status();
}

extern "C" int sa3_rmsnorm_quant_fused(const void* x, int x_dtype, void* out, int rows, int D, long long ldx,
                                       long long ldo, const float* gamma, float eps, const float* mod, long long ld_mod,
                                       int scale_off, int shift_off, int rows_per_batch, const int* row_batch,
                                       int out_dtype, float* amax, float* scale_out, float* row_r, unsigned int* barrier,
                                       void* stream) {
  if (!x || !out || !amax || !row_r || !barrier || rows <= 0 || D <= 0) return SA3_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(barrier) & 7) return SA3_ERR_ALIGN;
  const bool vec = aligned16(gamma) && (!mod || (aligned16(mod) && ld_mod % 4 == 0 && scale_off % 4 == 0 &&
                                                  shift_off % 4 == 0));
  int tab_batches = 1;
  if (mod) tab_batches = (!row_batch && rows_per_batch > 0 && (rows + rows_per_batch - 1) / rows_per_batch <= 2)
                             ? (rows + rows_per_batch - 1) / rows_per_batch
                             : 0;
  const bool out_ok = out_dtype == SA3_DT_E4M3 ? ((reinterpret_cast<uintptr_t>(out) & 7) == 0 && ldo % 8 == 0 && ldo >= D)
                                               : (out_dtype == SA3_DT_BF16 && aligned16(out) && ldo % 8 == 0 && ldo >= D);
  const bool fused = x_dtype == SA3_DT_F16 && D == 1536 && vec && tab_batches >= 1 && aligned16(x) && ldx % 8 == 0 &&
                     ldx >= D && out_ok;
  if (!fused) {
    // the two launches: max|y| (storing 1/rms per row), then the write pass
    int rc = sa3_rmsnorm_modulate(x, x_dtype, nullptr, rows, D, ldx, 0, gamma, eps, mod, ld_mod, scale_off, shift_off,
                                  rows_per_batch, row_batch, SA3_NORM_AMAX, out_dtype, nullptr, nullptr, amax, row_r,
                                  stream);
    if (rc) return rc;
    return sa3_rmsnorm_modulate(x, x_dtype, out, rows, D, ldx, ldo, gamma, eps, mod, ld_mod, scale_off, shift_off,
                                rows_per_batch, row_batch, SA3_NORM_WRITE, out_dtype, amax, scale_out, nullptr, row_r,
                                stream);
  }
  NormParams p;
  p.x = x;
  p.x_f32 = 0;
  p.x_f16 = 1;
  p.out = out;
  p.rows = rows;
  p.D = D;
  p.ldx = ldx;
  p.ldo = ldo;
  p.gamma = gamma;
  p.eps = eps;
  p.mod = mod;
  p.ld_mod = ld_mod;
  p.scale_off = scale_off;
  p.shift_off = shift_off;
  p.rows_per_batch = rows_per_batch;
  p.row_batch = nullptr;
  p.mode = SA3_NORM_WRITE;
  p.out_dtype = out_dtype;
  p.quant_amax = amax;
  p.scale_out = scale_out;
  p.amax_out = amax;
  p.row_r = row_r;
  const int smem = tab_batches * 2 * D * 4;
  int rc;
  if ((rc = ensure_smem(norm_fused_kernel<12>, 2 * 2 * 2048 * 4))) return rc;
  // every block of the grid must be resident at once for the barrier: at most the kernel's occupancy
  int dev = 0, sms = 0, per_sm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, norm_fused_kernel<12>, NORM_D_THREADS, smem) !=
          cudaSuccess ||
      per_sm <= 0 || sms <= 0)
    return SA3_ERR_LAUNCH;
  int grid = (rows + 7) / 8;
  if (grid > per_sm * sms) grid = per_sm * sms;
  launch_ex(norm_fused_kernel<12>, dim3(grid), dim3(NORM_D_THREADS), smem, reinterpret_cast<cudaStream_t>(stream), 1, p,
            tab_batches, barrier);
  return launch_status();
}

