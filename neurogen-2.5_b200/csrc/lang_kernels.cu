// Language-core kernels for sm_100a.
//
// Numerics contract: these kernels reproduce the reference CPU engine
// (src/native/CPUBackend.cpp, src/native/NeuralEngine.cpp) operation by
// operation in IEEE fp32 round-to-nearest:
//   * every dot product is accumulated strictly in increasing k order starting
//     from the bias (CPUBackend.cpp:14-17), one rounded multiply then one
//     rounded add per term -- no FMA contraction (this file is compiled with
//     -fmad=false and the inner loops use __fmul_rn/__fadd_rn explicitly);
//   * expressions are evaluated in the same association order as the C++;
//   * LayerNorm statistics are accumulated in fp64 (NeuralEngine.cpp:96-104);
//   * the input sigmoid and the feedback tanh return exactly the host C
//     library's values (expf, tanhf): a formula evaluated identically on host
//     and device, corrected by a table of the inputs where the library's
//     result differs (libm_match.cuh, math_tables.cpp).
// The result is bit-identical to the reference library.
#include "lang_kernels.h"

#include <cooperative_groups.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <cstdlib>
#include <stdexcept>
#include <string>

namespace cg = cooperative_groups;

namespace ngb {
namespace {

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
  unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async4(void *smem, const void *gmem) {
  unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------------------
// Projection, batch 1: one warp per 8 rows (a quarter of a 32-row panel); lanes
// 0-7 each own one row's sequential chain.  The quarter-panel's weights (32
// bytes per k) stream through a deep cp.async ring (GV_STAGES x GV_KC k) so
// that most of a row block is in flight at once and the chain, not L2
// latency, sets the time.
// ---------------------------------------------------------------------------
constexpr int GV_ROWS = 8, GV_KC = 64, GV_STAGES = 24;
constexpr int GV_STAGE_FLOATS = GV_KC * GV_ROWS + GV_KC;

__global__ void __launch_bounds__(32) k_gemv(ProjBatch pb) {
  extern __shared__ __align__(16) float gv[];
  const ProjArgs &a = pb.a[blockIdx.z];
  const int q = blockIdx.x, p = q >> 2, r0 = (q & 3) * GV_ROWS, lane = threadIdx.x;
  if (p * 32 >= a.M) return;
  const int m = p * 32 + r0 + lane;
  const float *x = a.x + (long)(a.xidx ? a.xidx[0] : 0) * a.ldx;
  const float *wq = a.wp + (size_t)p * a.K * 32 + r0;
  const int nch = (a.K + GV_KC - 1) / GV_KC;
  auto issue = [&](int ch) {
    if (ch < nch) {
      const int k0 = ch * GV_KC, kc = min(GV_KC, a.K - k0);
      float *ws = gv + (ch % GV_STAGES) * GV_STAGE_FLOATS;
      float *xs = ws + GV_KC * GV_ROWS;
      for (int i = lane; i < kc * 2; i += 32) // two 16-byte pieces per k
        cp_async16(ws + (i >> 1) * GV_ROWS + (i & 1) * 4, wq + (size_t)(k0 + (i >> 1)) * 32 + (i & 1) * 4);
      for (int i = lane; i < kc; i += 32) cp_async4(xs + i, x + k0 + i);
    }
    cp_async_commit();
  };
  for (int s = 0; s < GV_STAGES - 1; ++s) issue(s);
  float acc = (a.bias && lane < GV_ROWS && m < a.M) ? a.bias[m] : 0.f;
  for (int ch = 0; ch < nch; ++ch) {
    issue(ch + GV_STAGES - 1);
    cp_async_wait<GV_STAGES - 1>();
    __syncwarp();
    const float *ws = gv + (ch % GV_STAGES) * GV_STAGE_FLOATS;
    const float *xs = ws + GV_KC * GV_ROWS;
    if (lane < GV_ROWS) {
      const int kc = min(GV_KC, a.K - ch * GV_KC);
      if (kc == GV_KC) {
        // 16 independent products, then their 16 dependent adds: operand
        // loads and multiplies of the next group overlap this group's chain.
#pragma unroll
        for (int g = 0; g < GV_KC; g += 16) {
          float pr[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) pr[j] = __fmul_rn(ws[(g + j) * GV_ROWS + lane], xs[g + j]);
#pragma unroll
          for (int j = 0; j < 16; ++j) acc = __fadd_rn(acc, pr[j]);
        }
      } else {
        for (int k = 0; k < kc; ++k) acc = __fadd_rn(acc, __fmul_rn(ws[k * GV_ROWS + lane], xs[k]));
      }
    }
    __syncwarp();
  }
  if (lane < GV_ROWS && m < a.M) {
    if (a.addv) acc = __fadd_rn(acc, __fmul_rn(0.25f, a.addv[m]));
    a.y[m] = acc;
  }
}

// ---------------------------------------------------------------------------
// Projection, batch >= 2: CTA tile = one 32-row panel x BN sessions; each
// thread owns 4 rows x TN sessions (4*TN independent chains), so the FP32
// pipe stays busy while each chain waits on its previous add.  K is staged
// in 32-wide chunks through a 4-stage cp.async ring; the session operand is
// stored k-major so a thread's TN sessions are one vector load.  Every
// output is still one sequential chain over k (no split-K): results equal
// the batch-1 kernel's and the CPU's bit for bit.
// ---------------------------------------------------------------------------
constexpr int GM_KC = 32, GM_STAGES = 4;

template <int BN, int TN> __host__ __device__ constexpr int gemm_threads() { return 8 * (BN / TN); }
template <int BN> __host__ __device__ constexpr int gemm_stage_floats() { return GM_KC * 32 + GM_KC * BN; }

template <int TN> struct VecT;
template <> struct VecT<1> { using T = float; };
template <> struct VecT<2> { using T = float2; };
template <> struct VecT<4> { using T = float4; };

template <int TN>
__device__ __forceinline__ void load_x(const float *p, float (&x)[TN]) {
  const typename VecT<TN>::T v = *reinterpret_cast<const typename VecT<TN>::T *>(p);
  const float *f = reinterpret_cast<const float *>(&v);
#pragma unroll
  for (int s = 0; s < TN; ++s) x[s] = f[s];
}

// Packed pairs of fp32 (sm_100 f32x2): each lane of add.rn.f32x2 is one IEEE
// round-to-nearest fp32 add, so pairing two independent chains changes no
// bit.  Products stay scalar __fmul_rn: a packed multiply feeding a packed add
// is contracted into a fused multiply-add by the assembler, even written as
// mul.rn.f32x2 with the explicit rounding mode (both measured on B200: the
// projections stop being bit-identical), which would change the rounding.
typedef unsigned long long f32x2;
__device__ __forceinline__ f32x2 pack2(float lo, float hi) {
  f32x2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack2(f32x2 v, float &lo, float &hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ f32x2 add2(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

template <int BN, int TN>
__global__ void __launch_bounds__(gemm_threads<BN, TN>()) k_gemm(ProjBatch pb) {
  constexpr int NT = gemm_threads<BN, TN>(), STAGE = gemm_stage_floats<BN>();
  extern __shared__ __align__(16) float sm[];
  const ProjArgs &a = pb.a[blockIdx.z];
  const int p = blockIdx.x, b0 = blockIdx.y * BN;
  if (p * 32 >= a.M || b0 >= a.B) return;
  const int tid = threadIdx.x, tx = tid & 7, ty = tid >> 3;
  const int nch = (a.K + GM_KC - 1) / GM_KC;
  const float *wpan = a.wp + (size_t)p * a.K * 32;
  auto issue = [&](int ch) {
    if (ch < nch) {
      const int k0 = ch * GM_KC, kc = min(GM_KC, a.K - k0);
      float *ws = sm + (ch % GM_STAGES) * STAGE;
      float *xs = ws + GM_KC * 32;
      for (int i = tid; i < kc * 8; i += NT) cp_async16(ws + i * 4, wpan + (size_t)k0 * 32 + i * 4);
      for (int i = tid; i < BN * kc; i += NT) {
        const int sidx = i / kc, k = i - sidx * kc, b = b0 + sidx;
        if (b < a.B) cp_async4(xs + k * BN + sidx, a.x + (long)(a.xidx ? a.xidx[b] : b) * a.ldx + k0 + k);
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int s = 0; s < GM_STAGES - 1; ++s) issue(s);
  // acc[h][s]: rows (4tx + 2h, 4tx + 2h + 1) of session ty*TN + s.
  f32x2 acc[2][TN];
  {
    float init[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int m = p * 32 + tx * 4 + i;
      init[i] = (a.bias && m < a.M) ? a.bias[m] : 0.f;
    }
#pragma unroll
    for (int s = 0; s < TN; ++s) {
      acc[0][s] = pack2(init[0], init[1]);
      acc[1][s] = pack2(init[2], init[3]);
    }
  }
  for (int ch = 0; ch < nch; ++ch) {
    issue(ch + GM_STAGES - 1);
    cp_async_wait<GM_STAGES - 1>();
    __syncthreads();
    const float *ws = sm + (ch % GM_STAGES) * STAGE;
    const float *xs = ws + GM_KC * 32;
    const int kc = min(GM_KC, a.K - ch * GM_KC);
    auto step = [&](int k) {
      const float4 wv = *reinterpret_cast<const float4 *>(ws + k * 32 + tx * 4);
      float xr[TN];
      load_x<TN>(xs + k * BN + ty * TN, xr);
      f32x2 pr[2][TN];
#pragma unroll
      for (int s = 0; s < TN; ++s) {
        pr[0][s] = pack2(__fmul_rn(wv.x, xr[s]), __fmul_rn(wv.y, xr[s]));
        pr[1][s] = pack2(__fmul_rn(wv.z, xr[s]), __fmul_rn(wv.w, xr[s]));
      }
#pragma unroll
      for (int s = 0; s < TN; ++s) {
        acc[0][s] = add2(acc[0][s], pr[0][s]);
        acc[1][s] = add2(acc[1][s], pr[1][s]);
      }
    };
    if (kc == GM_KC) {
#pragma unroll
      for (int k = 0; k < GM_KC; ++k) step(k);
    } else {
      for (int k = 0; k < kc; ++k) step(k);
    }
    __syncthreads();
  }
#pragma unroll
  for (int s = 0; s < TN; ++s) {
    float r[4];
    unpack2(acc[0][s], r[0], r[1]);
    unpack2(acc[1][s], r[2], r[3]);
    const int b = b0 + ty * TN + s;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int m = p * 32 + tx * 4 + i;
      if (m < a.M && b < a.B) {
        float v = r[i];
        if (a.addv) v = __fadd_rn(v, __fmul_rn(0.25f, a.addv[(long)b * a.ldadd + m]));
        a.y[(long)b * a.ldy + m] = v;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Projection, small batch (2..64 sessions a launch column): 256 threads a CTA,
// thread (r, s) = (tid / BS, tid % BS) owns the one chain of row r0 + r and
// session b0 + s, so a 32-session tile gives a 768-row projection 768 warps.
// The CTA's 256/BS rows (a slice of one 32-row panel) and BS sessions stream
// through an 8-stage x 64-k cp.async ring, deep enough to cover L2 latency
// with few warps an SM.  Same sequential chain per output as every other
// projection kernel: results are bit-identical.
// ---------------------------------------------------------------------------
constexpr int SB_KC = 64, SB_STAGES = 8, SB_THREADS = 256;
template <int BS> __host__ __device__ constexpr int sb_rows() { return SB_THREADS / BS; }
template <int BS> __host__ __device__ constexpr int sb_stage_floats() { return SB_KC * (sb_rows<BS>() + BS); }

template <int BS>
__global__ void __launch_bounds__(SB_THREADS) k_gemm_sb(ProjBatch pb) {
  constexpr int RB = sb_rows<BS>(), STAGE = sb_stage_floats<BS>();
  extern __shared__ __align__(16) float sm[];
  const ProjArgs &a = pb.a[blockIdx.z];
  const int m0 = blockIdx.x * RB, b0 = blockIdx.y * BS;
  if (m0 >= a.M || b0 >= a.B) return;
  const int tid = threadIdx.x, r = tid / BS, s = tid % BS;
  const int p = m0 >> 5, r0 = m0 & 31; // panel and row offset inside it
  const float *wq = a.wp + (size_t)p * a.K * 32 + r0;
  const int nch = (a.K + SB_KC - 1) / SB_KC;
  auto issue = [&](int ch) {
    if (ch < nch) {
      const int k0 = ch * SB_KC, kc = min(SB_KC, a.K - k0);
      float *ws = sm + (ch % SB_STAGES) * STAGE;
      float *xs = ws + SB_KC * RB;
      constexpr int PIECES = RB / 4; // 16-byte pieces of a k's RB weights
      for (int i = tid; i < kc * PIECES; i += SB_THREADS) {
        const int k = i / PIECES, q = i - k * PIECES;
        cp_async16(ws + k * RB + q * 4, wq + (size_t)(k0 + k) * 32 + q * 4);
      }
      for (int i = tid; i < kc * BS; i += SB_THREADS) {
        const int sidx = i / kc, k = i - sidx * kc, b = b0 + sidx;
        if (b < a.B) cp_async4(xs + k * BS + sidx, a.x + (long)(a.xidx ? a.xidx[b] : b) * a.ldx + k0 + k);
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int st = 0; st < SB_STAGES - 1; ++st) issue(st);
  const int m = m0 + r, b = b0 + s;
  float acc = (a.bias && m < a.M) ? a.bias[m] : 0.f;
  for (int ch = 0; ch < nch; ++ch) {
    issue(ch + SB_STAGES - 1);
    cp_async_wait<SB_STAGES - 1>();
    __syncthreads();
    const float *ws = sm + (ch % SB_STAGES) * STAGE;
    const float *xs = ws + SB_KC * RB;
    const int kc = min(SB_KC, a.K - ch * SB_KC);
    if (kc == SB_KC) {
      // 16 independent products, then their 16 dependent adds.
#pragma unroll
      for (int g = 0; g < SB_KC; g += 16) {
        float pr[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) pr[j] = __fmul_rn(ws[(g + j) * RB + r], xs[(g + j) * BS + s]);
#pragma unroll
        for (int j = 0; j < 16; ++j) acc = __fadd_rn(acc, pr[j]);
      }
    } else {
      for (int k = 0; k < kc; ++k) acc = __fadd_rn(acc, __fmul_rn(ws[k * RB + r], xs[k * BS + s]));
    }
    __syncthreads();
  }
  if (m < a.M && b < a.B) {
    if (a.addv) acc = __fadd_rn(acc, __fmul_rn(0.25f, a.addv[(long)b * a.ldadd + m]));
    a.y[(long)b * a.ldy + m] = acc;
  }
}

template <int BS> size_t gemm_sb_smem() { return sizeof(float) * SB_STAGES * sb_stage_floats<BS>(); }

// ---------------------------------------------------------------------------
// Projection from row-major weights: CTA = RB rows x BS sessions; thread
// (r, s) owns the chains of row r for sessions s and s + BS/2, added as one
// add.rn.f32x2 pair (products stay scalar __fmul_rn).  Both operands stage
// along k in 16-byte cp.async pieces (weight rows W[m][k..], session inputs
// x[b][k..]) into rows padded to 68 floats, so each thread reads four k of
// its row and of its two sessions with three conflict-free 128-bit loads;
// the copy sources of each thread are fixed and computed once.  8-stage x
// 64-k ring.  Same sequential chain per output: bit-identical to the other
// projection kernels.  Needs K, ldx and the bases 16-byte aligned (checked by
// the launcher).
// ---------------------------------------------------------------------------
constexpr int RM_KC = 64, RM_STAGES = 8, RM_LD = RM_KC + 4;
template <int RB, int BS> __host__ __device__ constexpr int rm_stage_floats() { return (RB + BS) * RM_LD; }
template <int RB, int BS> __host__ __device__ constexpr int rm_threads() { return RB * BS / 2; }

template <int RB, int BS>
__global__ void __launch_bounds__(rm_threads<RB, BS>()) k_gemm_rm(ProjBatch pb) {
  constexpr int NT = rm_threads<RB, BS>(), STAGE = rm_stage_floats<RB, BS>(), HB = BS / 2;
  constexpr int PIECES = RM_KC / 4;                     // 16-byte pieces of a row's 64 k
  constexpr int WP = RB * PIECES / NT, XP = BS * PIECES / NT; // pieces a thread copies
  static_assert(RB * PIECES % NT == 0 && BS * PIECES % NT == 0, "tile");
  extern __shared__ __align__(16) float sm[];
  const ProjArgs &a = pb.a[blockIdx.z];
  const int m0 = blockIdx.x * RB, b0 = blockIdx.y * BS;
  if (m0 >= a.M || b0 >= a.B) return;
  const int tid = threadIdx.x, r = tid / HB, s = tid % HB;
  const int nch = (a.K + RM_KC - 1) / RM_KC;
  // Fixed copy assignment: piece i -> (row or session i / PIECES, piece i % PIECES).
  const float *wsrc[WP], *xsrc[XP];
  int wdst[WP], xdst[XP];
  bool wok[WP], xok[XP];
#pragma unroll
  for (int j = 0; j < WP; ++j) {
    const int i = tid + j * NT, rr = i / PIECES, q = i % PIECES;
    wok[j] = m0 + rr < a.M;
    wsrc[j] = a.wr + (size_t)(wok[j] ? m0 + rr : 0) * a.K + q * 4;
    wdst[j] = rr * RM_LD + q * 4;
  }
#pragma unroll
  for (int j = 0; j < XP; ++j) {
    const int i = tid + j * NT, ss = i / PIECES, q = i % PIECES, b = b0 + ss;
    xok[j] = b < a.B;
    xsrc[j] = a.x + (long)(xok[j] ? (a.xidx ? a.xidx[b] : b) : 0) * a.ldx + q * 4;
    xdst[j] = RB * RM_LD + ss * RM_LD + q * 4;
  }
  auto issue = [&](int ch) {
    if (ch < nch) {
      const int k0 = ch * RM_KC, kend = a.K - k0; // pieces at q*4 < kend are in range
      float *st = sm + (ch % RM_STAGES) * STAGE;
#pragma unroll
      for (int j = 0; j < WP; ++j)
        if (wok[j] && (wdst[j] % RM_LD) < kend) cp_async16(st + wdst[j], wsrc[j] + k0);
#pragma unroll
      for (int j = 0; j < XP; ++j)
        if (xok[j] && ((xdst[j] - RB * RM_LD) % RM_LD) < kend) cp_async16(st + xdst[j], xsrc[j] + k0);
    }
    cp_async_commit();
  };
#pragma unroll
  for (int st = 0; st < RM_STAGES - 1; ++st) issue(st);
  const int m = m0 + r, b_lo = b0 + s, b_hi = b0 + s + HB;
  const float bias = (a.bias && m < a.M) ? a.bias[m] : 0.f;
  f32x2 acc = pack2(bias, bias); // (session s, session s + BS/2)
  for (int ch = 0; ch < nch; ++ch) {
    issue(ch + RM_STAGES - 1);
    cp_async_wait<RM_STAGES - 1>();
    __syncthreads();
    const float *st = sm + (ch % RM_STAGES) * STAGE;
    const float *wrow = st + r * RM_LD, *xlo = st + RB * RM_LD + s * RM_LD, *xhi = xlo + HB * RM_LD;
    const int kc = min(RM_KC, a.K - ch * RM_KC);
    if (kc == RM_KC) {
#pragma unroll
      for (int q = 0; q < RM_KC / 4; ++q) {
        const float4 wv = *reinterpret_cast<const float4 *>(wrow + 4 * q);
        const float4 xl = *reinterpret_cast<const float4 *>(xlo + 4 * q);
        const float4 xh = *reinterpret_cast<const float4 *>(xhi + 4 * q);
        acc = add2(acc, pack2(__fmul_rn(wv.x, xl.x), __fmul_rn(wv.x, xh.x)));
        acc = add2(acc, pack2(__fmul_rn(wv.y, xl.y), __fmul_rn(wv.y, xh.y)));
        acc = add2(acc, pack2(__fmul_rn(wv.z, xl.z), __fmul_rn(wv.z, xh.z)));
        acc = add2(acc, pack2(__fmul_rn(wv.w, xl.w), __fmul_rn(wv.w, xh.w)));
      }
    } else {
      for (int k = 0; k < kc; ++k)
        acc = add2(acc, pack2(__fmul_rn(wrow[k], xlo[k]), __fmul_rn(wrow[k], xhi[k])));
    }
    __syncthreads();
  }
  float lo, hi;
  unpack2(acc, lo, hi);
  if (m < a.M) {
    if (b_lo < a.B) {
      if (a.addv) lo = __fadd_rn(lo, __fmul_rn(0.25f, a.addv[(long)b_lo * a.ldadd + m]));
      a.y[(long)b_lo * a.ldy + m] = lo;
    }
    if (b_hi < a.B) {
      if (a.addv) hi = __fadd_rn(hi, __fmul_rn(0.25f, a.addv[(long)b_hi * a.ldadd + m]));
      a.y[(long)b_hi * a.ldy + m] = hi;
    }
  }
}

template <int RB, int BS> size_t gemm_rm_smem() { return sizeof(float) * RM_STAGES * rm_stage_floats<RB, BS>(); }

// ---------------------------------------------------------------------------
// Projection, register-tiled (many sessions): 64 threads a CTA as an 8 x 8
// grid; thread (rt, st) owns TR rows x TS sessions, i.e. TR/2 x TS chains of
// row pairs (one add.rn.f32x2 each).  Per k a thread loads its TR weights
// (one shared-memory vector load) and TS inputs and issues TR*TS scalar
// __fmul_rn and TR*TS/2 packed adds, so the fp32 pipe, not shared-memory
// latency, sets the pace.  Weights stream from the 32-row panel layout by
// cp.async (RB = 8*TR rows of one panel are contiguous per k); the inputs are
// read 16 bytes at a time by the CTA's threads and stored transposed,
// [k][session], one chunk ahead of use.  Every output is still one
// sequential chain bias + w0*x0 + w1*x1 + ... : bits identical to every other
// projection kernel.
// ---------------------------------------------------------------------------
constexpr int RG_KC = 32, RG_STAGES = 4, RG_THREADS = 64, RG_AHEAD = 6;
template <int TR, int TS> __host__ __device__ constexpr int rg_rows() { return 8 * TR; }
template <int TR, int TS> __host__ __device__ constexpr int rg_sessions() { return 8 * TS; }
// Input tile row stride: sessions + 4 floats, so the transposing stores of the
// two k groups a warp writes land in different banks (and rows stay 16-byte aligned).
template <int TR, int TS> __host__ __device__ constexpr int rg_xld() { return 8 * TS + 4; }
template <int TR, int TS> __host__ __device__ constexpr int rg_stage_floats() {
  return RG_KC * (rg_rows<TR, TS>() + rg_xld<TR, TS>());
}
template <int TR, int TS> size_t gemm_rg_smem() { return sizeof(float) * RG_STAGES * rg_stage_floats<TR, TS>(); }

template <int N> __device__ __forceinline__ void lds_vec(const float *p, float (&v)[N]) {
  if constexpr (N == 4) {
    const float4 t = *reinterpret_cast<const float4 *>(p);
    v[0] = t.x, v[1] = t.y, v[2] = t.z, v[3] = t.w;
  } else if constexpr (N == 2) {
    const float2 t = *reinterpret_cast<const float2 *>(p);
    v[0] = t.x, v[1] = t.y;
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = p[i];
  }
}

template <int TR, int TS>
__global__ void __launch_bounds__(RG_THREADS) k_gemm_rg(ProjBatch pb) {
  constexpr int RB = rg_rows<TR, TS>(), BS = rg_sessions<TR, TS>(), XLD = rg_xld<TR, TS>();
  constexpr int STAGE = rg_stage_floats<TR, TS>();
  constexpr int WPIECES = RG_KC * RB / 4 / RG_THREADS; // 16-byte weight copies a thread, per chunk
  constexpr int XPIECES = BS * RG_KC / 4 / RG_THREADS; // 16-byte input loads a thread, per chunk
  static_assert(TR % 2 == 0 && 32 % RB == 0 && WPIECES >= 1 && XPIECES >= 1, "tile");
  extern __shared__ __align__(16) float sm[];
  const ProjArgs &a = pb.a[blockIdx.z];
  const int m0 = blockIdx.x * RB, b0 = blockIdx.y * BS;
  if (m0 >= a.M || b0 >= a.B) return;
  const int tid = threadIdx.x, rt = tid % 8, st = tid / 8;
  const int nch = (a.K + RG_KC - 1) / RG_KC;
  // Weights: panel rows m0 .. m0+RB-1 are RB contiguous floats for each k
  // (rows past M are the panel's zero padding).
  const float *wq = a.wp + (size_t)(m0 >> 5) * a.K * 32 + (m0 & 31);
  auto issue_w = [&](int ch) {
    if (ch < nch) {
      const int k0 = ch * RG_KC, kc = min(RG_KC, a.K - k0);
      float *ws = sm + (ch % RG_STAGES) * STAGE;
#pragma unroll
      for (int j = 0; j < WPIECES; ++j) {
        const int i = tid + j * RG_THREADS, k = i / (RB / 4), q = i % (RB / 4);
        if (k < kc) cp_async16(ws + k * RB + q * 4, wq + (size_t)(k0 + k) * 32 + q * 4);
      }
    }
    cp_async_commit();
  };
  // Inputs: piece i = (session i % BS, k quad i / BS); rows past B and k past
  // K read as zero.
  const float *xrow[XPIECES];
  int xs_sess[XPIECES], xs_kq[XPIECES];
#pragma unroll
  for (int j = 0; j < XPIECES; ++j) {
    const int i = tid + j * RG_THREADS, sidx = i % BS, b = b0 + sidx;
    xs_sess[j] = sidx;
    xs_kq[j] = i / BS;
    xrow[j] = b < a.B ? a.x + (long)(a.xidx ? a.xidx[b] : b) * a.ldx : nullptr;
  }
  float4 xr[XPIECES];
  auto load_x = [&](int ch) {
    const int k0 = ch * RG_KC;
#pragma unroll
    for (int j = 0; j < XPIECES; ++j) {
      const int k = k0 + 4 * xs_kq[j];
      xr[j] = (xrow[j] && k < a.K) ? *reinterpret_cast<const float4 *>(xrow[j] + k) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  auto store_x = [&](int ch) {
    float *xs = sm + (ch % RG_STAGES) * STAGE + RG_KC * RB;
#pragma unroll
    for (int j = 0; j < XPIECES; ++j) {
      float *d = xs + 4 * xs_kq[j] * XLD + xs_sess[j];
      d[0] = xr[j].x;
      d[XLD] = xr[j].y;
      d[2 * XLD] = xr[j].z;
      d[3 * XLD] = xr[j].w;
    }
  };
#pragma unroll
  for (int s = 0; s < RG_STAGES - 1; ++s) issue_w(s);
  load_x(0);
  store_x(0);
  if (nch > 1) load_x(1);

  // acc[p][s]: rows (m0 + TR*rt + 2p, +1) of session b0 + TS*st + s.
  f32x2 acc[TR / 2][TS];
#pragma unroll
  for (int p = 0; p < TR / 2; ++p) {
    const int m = m0 + TR * rt + 2 * p;
    const float lo = (a.bias && m < a.M) ? a.bias[m] : 0.f, hi = (a.bias && m + 1 < a.M) ? a.bias[m + 1] : 0.f;
#pragma unroll
    for (int s = 0; s < TS; ++s) acc[p][s] = pack2(lo, hi);
  }
  for (int ch = 0; ch < nch; ++ch) {
    cp_async_wait<RG_STAGES - 2>();
    __syncthreads();
    issue_w(ch + RG_STAGES - 1);
    if (ch + 1 < nch) store_x(ch + 1);
    if (ch + 2 < nch) load_x(ch + 2);
    const float *ws = sm + (ch % RG_STAGES) * STAGE + TR * rt;
    const float *xs = sm + (ch % RG_STAGES) * STAGE + RG_KC * RB + TS * st;
    auto fma_step = [&](const float (&w)[TR], const float (&x)[TS]) {
#pragma unroll
      for (int p = 0; p < TR / 2; ++p)
#pragma unroll
        for (int s = 0; s < TS; ++s)
          acc[p][s] = add2(acc[p][s], pack2(__fmul_rn(w[2 * p], x[s]), __fmul_rn(w[2 * p + 1], x[s])));
    };
    const int kc = min(RG_KC, a.K - ch * RG_KC);
    if (kc == RG_KC) {
      // Three-stage software pipeline over k: operands of step k + RG_AHEAD
      // are loaded and the products of step k + 1 formed while step k's
      // products are added, so neither shared-memory nor multiply latency
      // sits between two adds of a chain.
      float w[RG_AHEAD][TR], x[RG_AHEAD][TS];
      f32x2 pr[TR / 2][TS];
#pragma unroll
      for (int d = 0; d < RG_AHEAD; ++d) {
        lds_vec<TR>(ws + d * RB, w[d]);
        lds_vec<TS>(xs + d * XLD, x[d]);
      }
      auto products = [&](const float (&wv)[TR], const float (&xv)[TS]) {
#pragma unroll
        for (int p = 0; p < TR / 2; ++p)
#pragma unroll
          for (int s = 0; s < TS; ++s) pr[p][s] = pack2(__fmul_rn(wv[2 * p], xv[s]), __fmul_rn(wv[2 * p + 1], xv[s]));
      };
      products(w[0], x[0]);
#pragma unroll
      for (int k = 0; k < RG_KC; ++k) {
        f32x2 cur[TR / 2][TS];
#pragma unroll
        for (int p = 0; p < TR / 2; ++p)
#pragma unroll
          for (int s = 0; s < TS; ++s) cur[p][s] = pr[p][s];
        if (k + RG_AHEAD < RG_KC) {
          lds_vec<TR>(ws + (k + RG_AHEAD) * RB, w[k % RG_AHEAD]);
          lds_vec<TS>(xs + (k + RG_AHEAD) * XLD, x[k % RG_AHEAD]);
        }
        if (k + 1 < RG_KC) products(w[(k + 1) % RG_AHEAD], x[(k + 1) % RG_AHEAD]);
#pragma unroll
        for (int p = 0; p < TR / 2; ++p)
#pragma unroll
          for (int s = 0; s < TS; ++s) acc[p][s] = add2(acc[p][s], cur[p][s]);
      }
    } else {
      for (int k = 0; k < kc; ++k) {
        float w[TR], x[TS];
        lds_vec<TR>(ws + k * RB, w);
        lds_vec<TS>(xs + k * XLD, x);
        fma_step(w, x);
      }
    }
  }
#pragma unroll
  for (int p = 0; p < TR / 2; ++p)
#pragma unroll
    for (int s = 0; s < TS; ++s) {
      float r[2];
      unpack2(acc[p][s], r[0], r[1]);
      const int b = b0 + TS * st + s;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int m = m0 + TR * rt + 2 * p + i;
        if (m < a.M && b < a.B) {
          float v = r[i];
          if (a.addv) v = __fadd_rn(v, __fmul_rn(0.25f, a.addv[(long)b * a.ldadd + m]));
          a.y[(long)b * a.ldy + m] = v;
        }
      }
    }
}

template <int TR, int TS> void run_gemm_rg(const ProjBatch &pb, int max_m, int max_b, cudaStream_t s) {
  dim3 grid((max_m + rg_rows<TR, TS>() - 1) / rg_rows<TR, TS>(),
            (max_b + rg_sessions<TR, TS>() - 1) / rg_sessions<TR, TS>(), pb.count);
  k_gemm_rg<TR, TS><<<grid, RG_THREADS, gemm_rg_smem<TR, TS>(), s>>>(pb);
}

// Register-tiled operands usable: K, ldx and the input base 16-byte aligned
// (the weights come from the panel layout, always aligned).
bool rg_ok(const ProjBatch &pb) {
  for (int z = 0; z < pb.count; ++z) {
    const ProjArgs &a = pb.a[z];
    if (a.K % 4 || a.ldx % 4 || (reinterpret_cast<uintptr_t>(a.x) & 15)) return false;
  }
  return true;
}

template <int RB, int BS> void run_gemm_rm(const ProjBatch &pb, int max_m, int max_b, cudaStream_t s) {
  dim3 grid((max_m + RB - 1) / RB, (max_b + BS - 1) / BS, pb.count);
  k_gemm_rm<RB, BS><<<grid, rm_threads<RB, BS>(), gemm_rm_smem<RB, BS>(), s>>>(pb);
}

// Row-major operands usable: weights given, K, ldx and the bases 16-byte aligned.
bool rm_ok(const ProjBatch &pb) {
  for (int z = 0; z < pb.count; ++z) {
    const ProjArgs &a = pb.a[z];
    if (!a.wr || a.K % 4 || a.ldx % 4 || (reinterpret_cast<uintptr_t>(a.wr) & 15) ||
        (reinterpret_cast<uintptr_t>(a.x) & 15))
      return false;
  }
  return true;
}

template <int BS> void run_gemm_sb(const ProjBatch &pb, int max_m, int max_b, cudaStream_t s) {
  dim3 grid((max_m + sb_rows<BS>() - 1) / sb_rows<BS>(), (max_b + BS - 1) / BS, pb.count);
  k_gemm_sb<BS><<<grid, SB_THREADS, gemm_sb_smem<BS>(), s>>>(pb);
}

template <int BN, int TN> size_t gemm_smem() { return sizeof(float) * GM_STAGES * gemm_stage_floats<BN>(); }

template <int BN, int TN> void configure_gemm() {
  cudaFuncSetAttribute(k_gemm<BN, TN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_smem<BN, TN>());
}

template <int BN, int TN> void run_gemm(const ProjBatch &pb, int max_m, int max_b, cudaStream_t s) {
  dim3 grid((max_m + 31) / 32, (max_b + BN - 1) / BN, pb.count);
  k_gemm<BN, TN><<<grid, gemm_threads<BN, TN>(), gemm_smem<BN, TN>(), s>>>(pb);
}

// ---------------------------------------------------------------------------
// Recurrent ALIF tick: CTA = (column, SB sessions); 64 threads per session,
// one per unit.  The column's 64x64 weights are staged in shared memory with
// a padded row stride (65) so lanes reading different rows hit different
// banks; the previous trace of the column and of its two neighbours is
// staged too, because every unit reads all 64 traces of its column and the
// excitatory units read the same unit of the adjacent columns.
// ---------------------------------------------------------------------------
constexpr int TK_SB = 4, TK_LD = 65;

__global__ void __launch_bounds__(64 * TK_SB) k_tick(TickArgs a) {
  __shared__ float wt[64 * TK_LD];
  __shared__ float tr[TK_SB][3][64];
  const int col = blockIdx.x, s = threadIdx.x / 64, id = threadIdx.x % 64;
  const int b = blockIdx.y * TK_SB + s;
  const float *w = a.rec + (size_t)col * 4096;
  for (int i = threadIdx.x; i < 4096; i += 64 * TK_SB) wt[(i / 64) * TK_LD + i % 64] = w[i];
  if (b < a.B) {
    const float *t = a.tr_in + (long)b * a.tr_in_ld;
    tr[s][1][id] = t[col * 64 + id];
    tr[s][0][id] = col > 0 ? t[(col - 1) * 64 + id] : 0.f;
    tr[s][2][id] = col + 1 < a.c ? t[(col + 1) * 64 + id] : 0.f;
  }
  __syncthreads();
  if (b >= a.B) return;

  const bool exc = (a.tab.exc_mask >> id) & 1ull;
  // Input current (NeuralEngine.cpp:72-86).
  float current = exc ? .15f : .35f;
  const int ii = a.tab.in_idx[id], fi = a.tab.fb_idx[id];
  if (a.vin && ii >= 0) current = 3 * libm_match::sigmoid_host(a.vin[(long)b * a.c * a.tab.n_in + col * a.tab.n_in + ii], a.sig_tab, a.sig_neg_tab);
  if (fi >= 0) current = current + .5f * libm_match::tanh_host(a.fb[(long)b * a.c * a.tab.n_fb + col * a.tab.n_fb + fi], a.tanh_tab);

  // Recurrent input, sequential in the presynaptic index (CPUBackend.cpp:28-30).
  float recurrent = 0.f;
  const float *wr = wt + id * TK_LD;
#pragma unroll 16
  for (int j = 0; j < 64; ++j) recurrent = __fadd_rn(recurrent, __fmul_rn(wr[j], tr[s][1][j]));
  float neighbor = 0.f;
  if (exc) {
    if (col > 0) neighbor = neighbor + tr[s][0][id];
    if (col + 1 < a.c) neighbor = neighbor + tr[s][2][id];
  }

  float *st = a.state + (long)b * a.S + a.roff;
  const int n = a.n, i = col * 64 + id;
  const float V = st[i], adapt = st[2 * n + i], last = st[3 * n + i];
  const float cnt = st[4 * n + a.w + i];
  const float trace = tr[s][1][id];
  const float decay = exc ? .6f : .4f;
  const float voltage = decay * V + (1 - decay) * (current + recurrent + .08f * neighbor);
  const float spike = (voltage - (exc ? 1.f : .6f) - adapt >= 0 ? 1.f : 0.f) * (1 - last);
  const float v_out = voltage * (1 - spike);
  const float tr_out = .8f * trace + .2f * spike;
  st[i] = v_out;
  a.tr_out[(long)b * a.tr_out_ld + i] = tr_out;
  st[2 * n + i] = .98f * adapt + (exc ? .03f : 0.f) * spike;
  st[3 * n + i] = spike;
  st[4 * n + a.w + i] = cnt + spike;

  const unsigned fired = __ballot_sync(0xffffffffu, spike != 0.f);
  if ((threadIdx.x & 31) == 0 && fired) atomicAdd(a.spikes + (long)b * a.spikes_ld, __popc(fired));

  const int oi = a.tab.out_idx[id];
  if (a.feat && oi >= 0) {
    const int no = a.tab.n_out;
    float *f = a.feat + (long)b * (2 * a.c * no);
    f[col * no + oi] = v_out;
    f[a.c * no + col * no + oi] = tr_out;
  }
}

// ---------------------------------------------------------------------------
// All ticks of one region in one launch: a thread-block cluster of CL CTAs
// covers the region's c columns (CPC = c / CL each, weights in shared memory).
// A thread owns one unit of one column for SB sessions: its 64 recurrent
// weights are read 16 bytes at a time once per 4 k for all SB sessions, and
// each session's traces 16 bytes at a time (a broadcast to the column's 64
// threads).  Unit state stays in registers across ticks; each tick's traces
// go to a shared-memory ping-pong buffer, and the excitatory neighbour term
// reads the adjacent CTA's edge column through distributed shared memory after
// a cluster barrier.  Same arithmetic as k_tick, tick for tick: each session's
// recurrent input is still one sequential 64-term chain.
// ---------------------------------------------------------------------------
constexpr int TC_LD = 68; // weight row stride: 16-byte rows, 8 lanes' 16-byte loads hit distinct banks

template <int CPC, int SB>
__global__ void __launch_bounds__(64 * CPC) k_ticks_cluster(TickArgs a, int ticks) {
  extern __shared__ __align__(16) float tsm[];
  float *wt = tsm;                              // [CPC][64][TC_LD]
  float *trb = tsm + CPC * 64 * TC_LD;          // [2][SB][CPC][64]
  cg::cluster_group cluster = cg::this_cluster();
  const int g = blockIdx.x;                     // column group = rank in the cluster
  const int tid = threadIdx.x, id = tid & 63, cl = tid >> 6;
  const int col = g * CPC + cl, b0 = blockIdx.y * SB;
  {
    // The CTA's CPC x 4096 recurrent weights, 16-byte cp.async pieces.
    constexpr int NT = 64 * CPC, PIECES = CPC * 1024 / NT;
    const float *src = a.rec + (size_t)g * CPC * 4096;
#pragma unroll
    for (int u = 0; u < PIECES; ++u) {
      const int p = tid + u * NT, c = p >> 10, r = (p >> 4) & 63, q = p & 15;
      cp_async16(wt + (c * 64 + r) * TC_LD + q * 4, src + (size_t)p * 4);
    }
    cp_async_commit();
  }
  const bool exc = (a.tab.exc_mask >> id) & 1ull;
  const int n = a.n, i = col * 64 + id;
  float V[SB], trace[SB], adapt[SB], last[SB], cnt[SB], current[SB];
  // Input current (NeuralEngine.cpp:72-86): a unit takes the input sigmoid
  // (layer 4 E), the feedback tanh (layers 1, 5, 6) or neither; the library
  // corrections of all SB sessions are looked up together.
  const int ii = a.tab.in_idx[id], fi = a.tab.fb_idx[id];
  const bool sig = a.vin && ii >= 0, th = fi >= 0;
  float x[SB], z[SB];
  uint32_t key[SB];
  int which[SB]; // table: 0 sigmoid (x >= 0), 1 sigmoid (x < 0), 2 tanh, -1 none
#pragma unroll
  for (int s = 0; s < SB; ++s) {
    const int b = b0 + s;
    V[s] = trace[s] = adapt[s] = last[s] = cnt[s] = x[s] = 0.f;
    which[s] = -1;
    key[s] = 0u;
    if (b < a.B) {
      const float *st = a.state + (long)b * a.S + a.roff;
      V[s] = st[i];
      trace[s] = st[n + i];
      adapt[s] = st[2 * n + i];
      last[s] = st[3 * n + i];
      cnt[s] = st[4 * n + a.w + i];
      if (sig) x[s] = a.vin[(long)b * a.c * a.tab.n_in + col * a.tab.n_in + ii];
      else if (th) x[s] = a.fb[(long)b * a.c * a.tab.n_fb + col * a.tab.n_fb + fi];
      const uint32_t u = libm_match::bits_of(x[s]);
      which[s] = sig ? (int)(u >> 31) : th ? 2 : -1;
      key[s] = u & 0x7FFFFFFFu;
    }
  }
  // The formulas of all SB sessions side by side (independent FP64 chains).
  double ed[SB];
#pragma unroll
  for (int s = 0; s < SB; ++s) {
    ed[s] = 0.0;
    z[s] = sig ? libm_match::sigmoid_formula_d(x[s], ed[s]) : th ? libm_match::tanh_formula_d(x[s], ed[s]) : 0.f;
  }
  int dl[SB];
  libm_match::table_deltas<SB>(a.sig_tab, a.sig_neg_tab, a.tanh_tab, which, key, ed, dl);
#pragma unroll
  for (int s = 0; s < SB; ++s) {
    float cur = exc ? .15f : .35f;
    if (sig) cur = 3 * libm_match::add_ulps(z[s], dl[s]);
    else if (th) cur = cur + .5f * libm_match::add_ulps(z[s], dl[s]);
    current[s] = cur;
  }
  auto tr_at = [&](int buf, int ss, int cc) { return trb + ((buf * SB + ss) * CPC + cc) * 64; };
#pragma unroll
  for (int s = 0; s < SB; ++s) tr_at(0, s, cl)[id] = trace[s];
  cp_async_wait<0>();
  cluster.sync(); // weights and first traces visible
  const float decay = exc ? .6f : .4f;
  const float *wr = wt + (cl * 64 + id) * TC_LD;
  for (int t = 0; t < ticks; ++t) {
    const int cur = t & 1;
    float recurrent[SB];
#pragma unroll
    for (int s = 0; s < SB; ++s) recurrent[s] = 0.f;
    // Recurrent input, sequential in the presynaptic index (CPUBackend.cpp:28-30).
#pragma unroll 4
    for (int q = 0; q < 16; ++q) {
      const float4 w4 = *reinterpret_cast<const float4 *>(wr + 4 * q);
#pragma unroll
      for (int s = 0; s < SB; ++s) {
        const float4 t4 = *reinterpret_cast<const float4 *>(tr_at(cur, s, cl) + 4 * q);
        recurrent[s] = __fadd_rn(recurrent[s], __fmul_rn(w4.x, t4.x));
        recurrent[s] = __fadd_rn(recurrent[s], __fmul_rn(w4.y, t4.y));
        recurrent[s] = __fadd_rn(recurrent[s], __fmul_rn(w4.z, t4.z));
        recurrent[s] = __fadd_rn(recurrent[s], __fmul_rn(w4.w, t4.w));
      }
    }
#pragma unroll
    for (int s = 0; s < SB; ++s) {
      const bool live = b0 + s < a.B;
      float neighbor = 0.f;
      if (exc) {
        if (col > 0) {
          const float *left = cl > 0 ? tr_at(cur, s, cl - 1) : cluster.map_shared_rank(tr_at(cur, s, CPC - 1), g - 1);
          neighbor = neighbor + left[id];
        }
        if (col + 1 < a.c) {
          const float *right = cl + 1 < CPC ? tr_at(cur, s, cl + 1) : cluster.map_shared_rank(tr_at(cur, s, 0), g + 1);
          neighbor = neighbor + right[id];
        }
      }
      const float voltage = decay * V[s] + (1 - decay) * (current[s] + recurrent[s] + .08f * neighbor);
      const float spike = (voltage - (exc ? 1.f : .6f) - adapt[s] >= 0 ? 1.f : 0.f) * (1 - last[s]);
      V[s] = voltage * (1 - spike);
      trace[s] = .8f * trace[s] + .2f * spike;
      adapt[s] = .98f * adapt[s] + (exc ? .03f : 0.f) * spike;
      last[s] = spike;
      cnt[s] = cnt[s] + spike;
      tr_at(cur ^ 1, s, cl)[id] = trace[s];
      const unsigned fired = __ballot_sync(0xffffffffu, live && spike != 0.f);
      if ((tid & 31) == 0 && fired) atomicAdd(a.spikes + (long)(b0 + s) * a.spikes_ld, __popc(fired));
    }
    cluster.sync(); // new traces visible cluster-wide; old buffer free for reuse
  }
#pragma unroll
  for (int s = 0; s < SB; ++s) {
    const int b = b0 + s;
    if (b >= a.B) continue;
    float *st = a.state + (long)b * a.S + a.roff;
    st[i] = V[s];
    st[n + i] = trace[s];
    st[2 * n + i] = adapt[s];
    st[3 * n + i] = last[s];
    st[4 * n + a.w + i] = cnt[s];
    const int oi = a.tab.out_idx[id];
    if (a.feat && oi >= 0) {
      const int no = a.tab.n_out;
      float *f = a.feat + (long)b * (2 * a.c * no);
      f[col * no + oi] = V[s];
      f[a.c * no + col * no + oi] = trace[s];
    }
  }
}

template <int CPC, int SB> size_t ticks_cluster_smem() {
  return sizeof(float) * (CPC * 64 * TC_LD + 2 * SB * CPC * 64);
}

template <int CPC, int SB> void configure_ticks_cluster() {
  cudaFuncSetAttribute(k_ticks_cluster<CPC, SB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       (int)ticks_cluster_smem<CPC, SB>());
}

template <int CPC, int SB> cudaError_t run_ticks_cluster(const TickArgs &a, int ticks, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.c / CPC, (a.B + SB - 1) / SB, 1);
  cfg.blockDim = dim3(64 * CPC, 1, 1);
  cfg.dynamicSmemBytes = ticks_cluster_smem<CPC, SB>();
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = a.c / CPC;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_ticks_cluster<CPC, SB>, a, ticks);
}

template <int CPC> cudaError_t run_ticks_cluster_sb(const TickArgs &a, int ticks, int sb, cudaStream_t s) {
  switch (sb) {
  case 1: return run_ticks_cluster<CPC, 1>(a, ticks, s);
  case 2: return run_ticks_cluster<CPC, 2>(a, ticks, s);
  case 4: return run_ticks_cluster<CPC, 4>(a, ticks, s);
  default: return run_ticks_cluster<CPC, 8>(a, ticks, s);
  }
}

__global__ void k_copy_rows(const float *src, long src_ld, float *dst, long dst_ld, int n, int B) {
  const int b = blockIdx.y;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    dst[(long)b * dst_ld + i] = src[(long)b * src_ld + i];
}

// ---------------------------------------------------------------------------
// LayerNorm + memory update, one CTA per session (NeuralEngine.cpp:96-108).
// ---------------------------------------------------------------------------
constexpr int LN_T = 256;

__device__ double block_sum(double v, double *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double total = 0;
  if (threadIdx.x == 0) {
    for (int i = 0; i < LN_T / 32; ++i) total += red[i];
    red[LN_T / 32] = total;
  }
  __syncthreads();
  total = red[LN_T / 32];
  __syncthreads();
  return total;
}

__global__ void __launch_bounds__(LN_T) k_norm(NormArgs a) {
  __shared__ double red[LN_T / 32 + 1];
  const int b = blockIdx.x;
  const float *hr = a.hraw + (long)b * a.hraw_ld;
  double s = 0;
  for (int i = threadIdx.x; i < a.w; i += LN_T) s += (double)hr[i];
  const double mean = block_sum(s, red) / (double)a.w;
  double v = 0;
  for (int i = threadIdx.x; i < a.w; i += LN_T) {
    const double d = (double)hr[i] - mean;
    v += d * d;
  }
  const double var = block_sum(v, red);
  const float inv = (float)(1.0 / sqrt(var / (double)a.w + 1e-5));
  const float mf = (float)mean;
  float *h = a.h + (long)b * a.h_ld;
  float *mem = a.mem + (long)b * a.mem_ld;
  for (int i = threadIdx.x; i < a.w; i += LN_T) {
    const float y = (hr[i] - mf) * inv * a.norm_w[i] + a.norm_b[i];
    h[i] = y;
    if (a.h_hi) {
      const float hi = __uint_as_float(__float_as_uint(y) & 0xFFFFE000u);
      a.h_hi[(long)b * a.h_ld + i] = hi;
      a.h_lo[(long)b * a.h_ld + i] = __fsub_rn(y, hi);
    }
    const float d = a.decay[i];
    mem[i] = d * mem[i] + (1 - d) * y;
  }
}

__global__ void k_activity(const int *counts, int A, int R, int n, int T, float *act, int B) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const double denom = (double)n * (double)T;
  float total = 0.f;
  for (int adv = 0; adv < A; ++adv) {
    float sum = 0.f;
    for (int r = 0; r < R; ++r) sum = sum + (float)((double)counts[((long)b * A + adv) * R + r] / denom);
    sum = sum / (float)R;
    total = adv == 0 ? sum : total + sum;
  }
  act[b] = A == 1 ? total : total / (float)A;
}

} // namespace

void configure_lang_kernels() {
  configure_readout_tc();
  configure_ticks_cluster<4, 1>();
  configure_ticks_cluster<4, 2>();
  configure_ticks_cluster<4, 4>();
  configure_ticks_cluster<4, 8>();
  configure_ticks_cluster<2, 1>();
  configure_ticks_cluster<2, 2>();
  configure_ticks_cluster<2, 4>();
  configure_ticks_cluster<2, 8>();
  configure_ticks_cluster<1, 1>();
  configure_ticks_cluster<1, 2>();
  configure_ticks_cluster<1, 4>();
  configure_ticks_cluster<1, 8>();
  configure_gemm<8, 1>();
  configure_gemm<16, 2>();
  configure_gemm<32, 4>();
  configure_gemm<64, 4>();
  cudaFuncSetAttribute(k_gemm_rg<2, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_rg_smem<2, 2>());
  cudaFuncSetAttribute(k_gemm_rg<4, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_rg_smem<4, 2>());
  cudaFuncSetAttribute(k_gemm_rg<2, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_rg_smem<2, 4>());
  cudaFuncSetAttribute(k_gemm_rg<4, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_rg_smem<4, 4>());
  cudaFuncSetAttribute(k_gemm_rg<4, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_rg_smem<4, 3>());
  cudaFuncSetAttribute(k_gemm_rg<2, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_rg_smem<2, 3>());
  cudaFuncSetAttribute(k_gemm_rm<16, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_rm_smem<16, 8>());
  cudaFuncSetAttribute(k_gemm_rm<32, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_rm_smem<32, 8>());
  cudaFuncSetAttribute(k_gemm_sb<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_sb_smem<8>());
  cudaFuncSetAttribute(k_gemm_sb<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_sb_smem<16>());
  cudaFuncSetAttribute(k_gemm_sb<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_sb_smem<32>());
  cudaFuncSetAttribute(k_gemv, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       (int)(sizeof(float) * GV_STAGES * GV_STAGE_FLOATS));
}

void preload_lang_kernels() {
  cudaFuncAttributes fa;
  const void *kernels[] = {(const void *)k_gemv,
                           (const void *)k_gemm_rg<2, 2>,
                           (const void *)k_gemm_rg<4, 2>,
                           (const void *)k_gemm_rg<2, 4>,
                           (const void *)k_gemm_rg<4, 4>,
                           (const void *)k_gemm_rg<4, 3>,
                           (const void *)k_gemm_rg<2, 3>,
                           (const void *)k_gemm_rm<16, 8>,
                           (const void *)k_gemm_rm<32, 8>,
                           (const void *)k_gemm_sb<8>,
                           (const void *)k_gemm_sb<16>,
                           (const void *)k_gemm_sb<32>,
                           (const void *)k_gemm<8, 1>,
                           (const void *)k_gemm<16, 2>,
                           (const void *)k_gemm<32, 4>,
                           (const void *)k_gemm<64, 4>,
                           (const void *)k_tick,
                           (const void *)k_ticks_cluster<4, 1>,
                           (const void *)k_ticks_cluster<4, 2>,
                           (const void *)k_ticks_cluster<4, 4>,
                           (const void *)k_ticks_cluster<4, 8>,
                           (const void *)k_ticks_cluster<2, 1>,
                           (const void *)k_ticks_cluster<2, 2>,
                           (const void *)k_ticks_cluster<2, 4>,
                           (const void *)k_ticks_cluster<2, 8>,
                           (const void *)k_ticks_cluster<1, 1>,
                           (const void *)k_ticks_cluster<1, 2>,
                           (const void *)k_ticks_cluster<1, 4>,
                           (const void *)k_ticks_cluster<1, 8>,
                           (const void *)k_copy_rows,
                           (const void *)k_norm,
                           (const void *)k_activity};
  for (const void *k : kernels) cudaFuncGetAttributes(&fa, k);
  cudaFuncGetAttributes(&fa, readout_tc_kernel());
}

void launch_projections(const ProjBatch &pb, cudaStream_t s) {
  int max_m = 0, max_b = 0;
  for (int z = 0; z < pb.count; ++z) {
    max_m = max(max_m, pb.a[z].M);
    max_b = max(max_b, pb.a[z].B);
  }
  if (max_m <= 0 || max_b <= 0) return;
  if (max_b == 1) {
    dim3 grid(((max_m + 31) / 32) * 4, 1, pb.count);
    k_gemv<<<grid, 32, sizeof(float) * GV_STAGES * GV_STAGE_FLOATS, s>>>(pb);
    return;
  }
  // Most independent chains per thread that still gives every SM sub-partition
  // (148 SMs x 4) a warp; else the finest tile.
  const long panels = (max_m + 31) / 32;
  auto warps = [&](int bn, int threads) { return panels * ((max_b + bn - 1) / bn) * (threads / 32) * pb.count; };
  const long want = 148 * 4;
  // NEUROGEN_PROJ_TILE = 8 | 16 | 32 | 64 forces one session tile (tests of
  // every tile shape); results do not depend on the tile.
  static const int forced = [] {
    const char *v = std::getenv("NEUROGEN_PROJ_TILE");
    return v ? std::atoi(v) : 0;
  }();
  // NEUROGEN_PROJ_SMALL = 8 | 16 | 32 forces the small-batch kernel's session
  // tile the same way.
  static const int forced_small = [] {
    const char *v = std::getenv("NEUROGEN_PROJ_SMALL");
    return v ? std::atoi(v) : 0;
  }();
  // NEUROGEN_PROJ_ROWMAJOR = 16 | 32 forces the row-major kernel with that
  // many rows a CTA (when its operands qualify).
  static const int forced_rm = [] {
    const char *v = std::getenv("NEUROGEN_PROJ_ROWMAJOR");
    return v ? std::atoi(v) : 0;
  }();
  // NEUROGEN_PROJ_REG = 22 | 42 | 24 | 44 forces the register-tiled kernel
  // with that many rows and sessions a thread (when its operands qualify).
  static const int forced_rg = [] {
    const char *v = std::getenv("NEUROGEN_PROJ_REG");
    return v ? std::atoi(v) : 0;
  }();
  if (forced_rg > 0 && rg_ok(pb)) {
    switch (forced_rg) {
    case 42: return run_gemm_rg<4, 2>(pb, max_m, max_b, s);
    case 24: return run_gemm_rg<2, 4>(pb, max_m, max_b, s);
    case 44: return run_gemm_rg<4, 4>(pb, max_m, max_b, s);
    case 43: return run_gemm_rg<4, 3>(pb, max_m, max_b, s);
    case 23: return run_gemm_rg<2, 3>(pb, max_m, max_b, s);
    default: return run_gemm_rg<2, 2>(pb, max_m, max_b, s);
    }
  }
  if (forced_rm && rm_ok(pb)) {
    if (forced_rm == 32) return run_gemm_rm<32, 8>(pb, max_m, max_b, s);
    return run_gemm_rm<16, 8>(pb, max_m, max_b, s);
  }
  switch (forced_small) {
  case 8: return run_gemm_sb<8>(pb, max_m, max_b, s);
  case 16: return run_gemm_sb<16>(pb, max_m, max_b, s);
  case 32: return run_gemm_sb<32>(pb, max_m, max_b, s);
  default: break;
  }
  switch (forced) {
  case 8: return run_gemm<8, 1>(pb, max_m, max_b, s);
  case 16: return run_gemm<16, 2>(pb, max_m, max_b, s);
  case 32: return run_gemm<32, 4>(pb, max_m, max_b, s);
  case 64: return run_gemm<64, 4>(pb, max_m, max_b, s);
  default: break;
  }
  // Register tiles when they give every SM sub-partition (148 x 4) at least
  // one warp: 4 rows x 2 sessions a thread, else 2 x 2 (BC-250, 256 sessions:
  // feedback 4x2, input 2x2, output 4x2; 122 K -> 160 K tokens/s).
  // NEUROGEN_PROJ_REG=-1 keeps the row-major kernel at every size.
  if (forced_rg == 0 && rg_ok(pb)) {
    auto rg_warps = [&](int rows, int sessions) {
      long w = 0;
      for (int z = 0; z < pb.count; ++z)
        w += long((pb.a[z].M + rows - 1) / rows) * ((pb.a[z].B + sessions - 1) / sessions) * (RG_THREADS / 32);
      return w;
    };
    if (rg_warps(rg_rows<4, 2>(), rg_sessions<4, 2>()) >= want) return run_gemm_rg<4, 2>(pb, max_m, max_b, s);
    if (rg_warps(rg_rows<2, 2>(), rg_sessions<2, 2>()) >= want) return run_gemm_rg<2, 2>(pb, max_m, max_b, s);
  }
  // Row-major operands (the engine's default): 16 rows x 8 sessions a CTA,
  // measured fastest at every batch on BC-250 (32 / 64 / 128 / 256 sessions:
  // 44.0 K / 71.0 K / 88.3 K / 104.4 K tokens/s, against 36.8 K / 50.4 K /
  // 74.6 K / 92.7 K with the panel kernels).
  if (rm_ok(pb)) return run_gemm_rm<16, 8>(pb, max_m, max_b, s);
  // Up to 64 sessions: one chain a thread (small-batch kernel) on whole
  // 32-row panels x 8 sessions, so each session input is staged once a panel.
  if (max_b <= 64) return run_gemm_sb<8>(pb, max_m, max_b, s);
  if (max_b > 32 && warps(64, gemm_threads<64, 4>()) >= want) run_gemm<64, 4>(pb, max_m, max_b, s);
  else if (max_b > 16 && warps(32, gemm_threads<32, 4>()) >= want) run_gemm<32, 4>(pb, max_m, max_b, s);
  else if (max_b > 8 && warps(16, gemm_threads<16, 2>()) >= want) run_gemm<16, 2>(pb, max_m, max_b, s);
  else run_gemm<8, 1>(pb, max_m, max_b, s);
}

void launch_projection(const ProjArgs &a, cudaStream_t s) {
  ProjBatch pb{};
  pb.a[0] = a;
  pb.count = 1;
  launch_projections(pb, s);
}

bool launch_ticks_cluster(const TickArgs &a, int ticks, cudaStream_t s) {
  // Columns per CTA so that the cluster (c / CPC CTAs) is at most 8 wide.
  const int cpc = (a.c % 4 == 0 && a.c / 4 <= 8) ? 4 : (a.c % 2 == 0 && a.c / 2 <= 8) ? 2 : a.c <= 8 ? 1 : 0;
  if (!cpc) return false;
  // Sessions a thread: the most (up to 8) that still give ~1.6 CTAs a SM
  // (BC-250: 8 at 256 sessions, 1 at 32; measured best at both).
  // NEUROGEN_TICK_SB = 1 | 2 | 4 | 8 forces one; results do not depend on it.
  int sb = 8;
  while (sb > 1 && long(a.c / cpc) * ((a.B + sb - 1) / sb) < 240) sb >>= 1;
  if (const char *v = std::getenv("NEUROGEN_TICK_SB")) sb = std::atoi(v);
  cudaError_t e;
  if (cpc == 4) e = run_ticks_cluster_sb<4>(a, ticks, sb, s);
  else if (cpc == 2) e = run_ticks_cluster_sb<2>(a, ticks, sb, s);
  else e = run_ticks_cluster_sb<1>(a, ticks, sb, s);
  if (e != cudaSuccess) throw std::runtime_error(std::string("cluster tick launch: ") + cudaGetErrorString(e));
  return true;
}

void launch_tick(const TickArgs &a, cudaStream_t s) {
  dim3 grid(a.c, (a.B + TK_SB - 1) / TK_SB);
  k_tick<<<grid, 64 * TK_SB, 0, s>>>(a);
}

void launch_copy_rows(const float *src, long src_ld, float *dst, long dst_ld, int n, int B,
                      cudaStream_t s) {
  dim3 grid((n + 255) / 256, B);
  k_copy_rows<<<grid, 256, 0, s>>>(src, src_ld, dst, dst_ld, n, B);
}

void launch_norm(const NormArgs &a, cudaStream_t s) { k_norm<<<a.B, LN_T, 0, s>>>(a); }

void launch_activity(const int *counts, int A, int R, int n, int T, float *act, int B,
                     cudaStream_t s) {
  k_activity<<<(B + 127) / 128, 128, 0, s>>>(counts, A, R, n, T, act, B);
}

} // namespace ngb
