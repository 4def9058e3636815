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
//   * exp is evaluated in fp64 and rounded once to fp32, which equals glibc's
//     expf except in rare ties; tanh uses the identity
//       tanh(x) = 1 - 2/(expm1(2x)+2)           for |x| >= 1,
//       tanh(x) = -expm1(-2x)/(expm1(-2x)+2)     for |x| <  1,
//     evaluated in fp32 around a once-rounded fp64 expm1, which is the form the
//     host libm evaluates (it agrees with glibc 2.39 tanhf on ~98% of inputs,
//     1 ulp otherwise).
// The result is bit-identical to the reference library except where a libm
// result differs by an ulp; the parity tests quantify that.
#include "lang_kernels.h"

#include <cuda_runtime.h>
#include <cstdint>

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

__device__ __forceinline__ float host_expf(float x) { return (float)exp((double)x); }

// 1 / (1 + exp(-x)) as NeuralEngine.cpp:9.
__device__ __forceinline__ float host_sigmoid(float x) {
  return __fdiv_rn(1.f, __fadd_rn(1.f, host_expf(-x)));
}

// tanh via the expm1 identity (see file header).
__device__ __forceinline__ float host_tanh(float x) {
  const float ax = fabsf(x);
  float z;
  if (ax >= 22.f) {
    z = 1.f;
  } else if (ax >= 1.f) {
    const float t = (float)expm1((double)(2.f * ax));
    z = __fsub_rn(1.f, __fdiv_rn(2.f, __fadd_rn(t, 2.f)));
  } else if (ax < 0x1p-55f) {
    z = ax;
  } else {
    const float t = (float)expm1((double)(-2.f * ax));
    z = __fdiv_rn(-t, __fadd_rn(t, 2.f));
  }
  return x < 0.f ? -z : z;
}

// ---------------------------------------------------------------------------
// Projection, batch 1: one warp per 32-row panel, one lane per row.  The
// panel's [K][32] weights stream through an 8-stage cp.async ring so the
// strictly sequential accumulation chain never waits on L2.
// ---------------------------------------------------------------------------
constexpr int GV_KC = 32, GV_STAGES = 8;

__global__ void __launch_bounds__(32) k_gemv(ProjArgs a) {
  __shared__ __align__(16) float ws[GV_STAGES][GV_KC * 32];
  __shared__ __align__(16) float xs[GV_STAGES][GV_KC];
  const int p = blockIdx.x, b = blockIdx.y, lane = threadIdx.x;
  const int m = p * 32 + lane;
  const float *x = a.x + (long)(a.xidx ? a.xidx[b] : b) * a.ldx;
  const float *wpan = a.wp + (size_t)p * a.K * 32;
  const int nch = (a.K + GV_KC - 1) / GV_KC;
  auto issue = [&](int ch) {
    if (ch < nch) {
      const int k0 = ch * GV_KC, kc = min(GV_KC, a.K - k0);
      const float *src = wpan + (size_t)k0 * 32;
      float *dst = ws[ch % GV_STAGES];
      for (int i = lane; i < kc * 8; i += 32) cp_async16(dst + i * 4, src + i * 4);
      for (int i = lane; i < kc; i += 32) cp_async4(&xs[ch % GV_STAGES][i], x + k0 + i);
    }
    cp_async_commit();
  };
#pragma unroll
  for (int s = 0; s < GV_STAGES - 1; ++s) issue(s);
  float acc = (a.bias && m < a.M) ? a.bias[m] : 0.f;
  for (int ch = 0; ch < nch; ++ch) {
    issue(ch + GV_STAGES - 1);
    cp_async_wait<GV_STAGES - 1>();
    __syncwarp();
    const float *w = ws[ch % GV_STAGES];
    const float *xv = xs[ch % GV_STAGES];
    const int kc = min(GV_KC, a.K - ch * GV_KC);
    if (kc == GV_KC) {
#pragma unroll
      for (int k = 0; k < GV_KC; ++k) acc = __fadd_rn(acc, __fmul_rn(w[k * 32 + lane], xv[k]));
    } else {
      for (int k = 0; k < kc; ++k) acc = __fadd_rn(acc, __fmul_rn(w[k * 32 + lane], xv[k]));
    }
    __syncwarp();
  }
  if (m < a.M) {
    if (a.addv) acc = __fadd_rn(acc, __fmul_rn(0.25f, a.addv[(long)b * a.ldadd + m]));
    a.y[(long)b * a.ldy + m] = acc;
  }
}

// ---------------------------------------------------------------------------
// Projection, batch >= 2: CTA tile BM rows x BN sessions, 4 rows x TN
// sessions per thread, K staged in KC chunks through a cp.async ring.  Each
// output is still one sequential chain over k (no split-K), so the result is
// identical to the batch-1 kernel and to the CPU.
// ---------------------------------------------------------------------------
constexpr int GM_KC = 32, GM_STAGES = 4, GM_BM = 64;

template <int BN, int TN>
__global__ void __launch_bounds__((GM_BM / 4) * (BN / TN)) k_gemm(ProjArgs a) {
  constexpr int BM = GM_BM, KC = GM_KC, TX = BM / 4, TY = BN / TN, NT = TX * TY;
  constexpr int XLD = KC + 4;
  constexpr int WS = KC * BM, XS = BN * XLD, STAGE = WS + XS;
  extern __shared__ __align__(16) float sm[];
  const int tid = threadIdx.x, tx = tid % TX, ty = tid / TX;
  const int m0 = blockIdx.x * BM, b0 = blockIdx.y * BN;
  const int P = (a.M + 31) / 32;
  const int nch = (a.K + KC - 1) / KC;
  auto issue = [&](int ch) {
    if (ch < nch) {
      const int k0 = ch * KC, kc = min(KC, a.K - k0);
      float *ws = sm + (ch % GM_STAGES) * STAGE;
      float *xs = ws + WS;
      const int wpieces = (BM / 32) * kc * 8;
      for (int i = tid; i < wpieces; i += NT) {
        const int q = i / (kc * 8), r = i % (kc * 8), k = r / 8, j4 = r % 8;
        const int pan = m0 / 32 + q;
        if (pan < P)
          cp_async16(ws + k * BM + q * 32 + j4 * 4, a.wp + ((size_t)pan * a.K + k0 + k) * 32 + j4 * 4);
      }
      for (int i = tid; i < BN * kc; i += NT) {
        const int s = i / kc, k = i % kc, b = b0 + s;
        if (b < a.B) {
          const float *xr = a.x + (long)(a.xidx ? a.xidx[b] : b) * a.ldx;
          cp_async4(xs + s * XLD + k, xr + k0 + k);
        }
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int s = 0; s < GM_STAGES - 1; ++s) issue(s);
  float acc[4][TN];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + tx * 4 + i;
    const float init = (a.bias && m < a.M) ? a.bias[m] : 0.f;
#pragma unroll
    for (int s = 0; s < TN; ++s) acc[i][s] = init;
  }
  for (int ch = 0; ch < nch; ++ch) {
    issue(ch + GM_STAGES - 1);
    cp_async_wait<GM_STAGES - 1>();
    __syncthreads();
    const float *ws = sm + (ch % GM_STAGES) * STAGE;
    const float *xs = ws + WS;
    const int kc = min(KC, a.K - ch * KC);
    for (int k = 0; k < kc; ++k) {
      const float4 wv = *reinterpret_cast<const float4 *>(ws + k * BM + tx * 4);
      const float w4[4] = {wv.x, wv.y, wv.z, wv.w};
      float xr[TN];
#pragma unroll
      for (int s = 0; s < TN; ++s) xr[s] = xs[(ty * TN + s) * XLD + k];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int s = 0; s < TN; ++s) acc[i][s] = __fadd_rn(acc[i][s], __fmul_rn(w4[i], xr[s]));
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + tx * 4 + i;
#pragma unroll
    for (int s = 0; s < TN; ++s) {
      const int b = b0 + ty * TN + s;
      if (m < a.M && b < a.B) {
        float v = acc[i][s];
        if (a.addv) v = __fadd_rn(v, __fmul_rn(0.25f, a.addv[(long)b * a.ldadd + m]));
        a.y[(long)b * a.ldy + m] = v;
      }
    }
  }
}

template <int BN, int TN> size_t gemm_smem() {
  return sizeof(float) * GM_STAGES * (GM_KC * GM_BM + BN * (GM_KC + 4));
}

template <int BN, int TN> void configure_gemm() {
  cudaFuncSetAttribute(k_gemm<BN, TN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_smem<BN, TN>());
}

template <int BN, int TN> void run_gemm(const ProjArgs &a, cudaStream_t s) {
  const size_t smem = gemm_smem<BN, TN>();
  dim3 grid((a.M + GM_BM - 1) / GM_BM, (a.B + BN - 1) / BN);
  k_gemm<BN, TN><<<grid, (GM_BM / 4) * (BN / TN), smem, s>>>(a);
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
  if (a.vin && ii >= 0) current = 3 * host_sigmoid(a.vin[(long)b * a.c * a.tab.n_in + col * a.tab.n_in + ii]);
  if (fi >= 0) current = current + .5f * host_tanh(a.fb[(long)b * a.c * a.tab.n_fb + col * a.tab.n_fb + fi]);

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
  configure_gemm<16, 1>();
  configure_gemm<32, 2>();
  configure_gemm<64, 4>();
}

void launch_projection(const ProjArgs &a, cudaStream_t s) {
  if (a.B <= 0 || a.M <= 0) return;
  if (a.B == 1) {
    dim3 grid((a.M + 31) / 32, 1);
    k_gemv<<<grid, 32, 0, s>>>(a);
    return;
  }
  // Smallest session tile that still gives every SM a CTA, else the widest.
  const long mt = (a.M + GM_BM - 1) / GM_BM;
  const int sms = 148;
  if (a.B <= 16 || mt * ((a.B + 31) / 32) < sms) run_gemm<16, 1>(a, s);
  else if (mt * ((a.B + 63) / 64) < sms) run_gemm<32, 2>(a, s);
  else run_gemm<64, 4>(a, s);
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
