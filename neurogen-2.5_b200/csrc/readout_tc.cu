// Token readout on the 5th-generation tensor cores:
//   logits[b][v] = bias[v] + sum_k h[b][k] * W[v][k]
// (reference: the language model head, neurogen/language/model.py head
// Linear(width, 264), evaluated by the native engine in
// src/native/engine/NeuralEngine.cpp as a sequential fp32 dot product).
//
// The tensor cores read fp32 operands as tf32 (10 explicit mantissa bits), so
// every operand x is split as hi = x with the low 13 mantissa bits cleared
// (exactly a tf32 value) and lo = x - hi (exact in fp32, read as tf32), and
//   h.W ~= h_hi.W_hi + (h_lo.W_hi + h_hi.W_lo)
// with the small terms in their own TMEM accumulator.  The k range is split
// into up to kSegs segments with separate accumulators, summed in fp32 in the
// epilogue (bias, main segments, then correction segments, a fixed order), so
// each accumulator takes few tensor-core additions.  The result is within a
// few 1e-6 of the vector scale of the sequential fp32 sum; it is deterministic
// but not bit-identical to it (the SIMT projection, k_gemm_rm / k_gemv, is).
//
// CTA: 128 sessions (TMEM lanes) x 32 vocabulary rows (TMEM columns), 128
// threads.  Per 32-wide k chunk, thread 0 loads the fp32 tiles of h and W by
// TMA (SWIZZLE_128B, kRaw stages deep); all threads split them element by
// element into hi / lo operand tiles of the same swizzled K-major layout
// (kOps stages); thread 0 issues the 12 MMAs of the chunk (4 k-steps x 3
// terms, M=128 N=32 K=8) and commits them to the stage's mbarrier.  Every
// mbarrier wait is bounded: on a timeout the kernel sets *err, stops issuing,
// waits (bounded) for work in flight, frees its TMEM and returns.
#include "lang_kernels.h"

#include <cuda.h>
#include <cstdlib>
#include <cstring>

namespace ngb {
namespace {

constexpr int kBM = 128, kBN = 32, kKC = 32;   // sessions, vocab rows, k per chunk
constexpr int kRaw = 4, kOps = 2, kSegs = 4;   // raw / operand stages, k segments
constexpr int kThreads = 128;
constexpr int kTmemCols = 256;                 // kSegs main + kSegs correction accumulators of kBN
constexpr uint32_t kTileA = kBM * kKC * 4, kTileB = kBN * kKC * 4; // 16 KB, 4 KB
constexpr uint32_t kRawBytes = kTileA + kTileB;                    // one raw stage
constexpr uint32_t kOpBytes = 2 * (kTileA + kTileB);               // hi + lo of both
constexpr size_t kSmemBytes = 1024 + kRaw * kRawBytes + kOps * kOpBytes + 256;
constexpr long kWaitLimit = 1L << 24;

// Instruction descriptor, kind::tf32: D f32 (bits 4-5 = 1), A and B tf32
// (bits 7-9, 10-12 = 2), both K-major (bits 15, 16 = 0), N >> 3 at bits
// 17-22, M >> 4 at bits 24-28.
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(kBN >> 3) << 17) |
                            (uint32_t(kBM >> 4) << 24);

// Shared-memory matrix descriptor of a K-major SWIZZLE_128B tile whose rows
// are 128 bytes apart (8-row atoms of 1024 bytes): start address >> 4 at bits
// 0-13, leading offset 16 B (unused by this layout) at 16-29, stride offset
// 1024 B >> 4 at 32-45, descriptor version 1 at bit 46, layout 2 (128-byte
// swizzle) at bits 61-63.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return uint64_t((saddr & 0x3FFFF) >> 4) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n\t.reg .pred p;\n\t"
               "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
               "selp.u32 %0, 1, 0, p;\n\t}"
               : "=r"(ok)
               : "r"(bar), "r"(parity)
               : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  for (long i = 0; i < kWaitLimit; ++i)
    if (mbar_try(bar, parity)) return true;
  return false;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar) {
  asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
               ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
               : "memory");
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
  asm volatile("{\n\t.reg .pred p;\n\t"
               "setp.ne.b32 p, %4, 0;\n\t"
               "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
               ::"r"(d_tmem), "l"(a), "l"(b), "r"(kIdesc), "r"(accumulate)
               : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// 32 consecutive fp32 TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld32(uint32_t addr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 "
               "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
               "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                 "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
                 "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
                 "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
                 "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
               : "r"(addr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}

__device__ __forceinline__ float4 tf32_hi(float4 x) {
  return make_float4(__uint_as_float(__float_as_uint(x.x) & 0xFFFFE000u),
                     __uint_as_float(__float_as_uint(x.y) & 0xFFFFE000u),
                     __uint_as_float(__float_as_uint(x.z) & 0xFFFFE000u),
                     __uint_as_float(__float_as_uint(x.w) & 0xFFFFE000u));
}

__device__ __forceinline__ void split_tile(const float4 *raw, float4 *hi, float4 *lo, int n4, int tid) {
  for (int i = tid; i < n4; i += kThreads) {
    const float4 x = raw[i], h = tf32_hi(x);
    hi[i] = h;
    lo[i] = make_float4(__fsub_rn(x.x, h.x), __fsub_rn(x.y, h.y), __fsub_rn(x.z, h.z), __fsub_rn(x.w, h.w));
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    k_readout_tc(const __grid_constant__ CUtensorMap tm_h, const __grid_constant__ CUtensorMap tm_w,
                 ReadoutArgs a) {
  extern __shared__ uint8_t smem_raw[];
  // 128-byte swizzled tiles start on 1024-byte boundaries of the shared window.
  uint8_t *base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t *raw = base;                              // kRaw x [A 16 KB][B 4 KB]
  uint8_t *ops = raw + kRaw * kRawBytes;            // kOps x [A hi][A lo][B hi][B lo]
  uint64_t *bars = reinterpret_cast<uint64_t *>(ops + kOps * kOpBytes); // raw_full[kRaw], mma_done[kOps]
  volatile uint32_t *tmem_slot = reinterpret_cast<volatile uint32_t *>(bars + kRaw + kOps);
  volatile int *abort_s = reinterpret_cast<volatile int *>(tmem_slot + 1);
  volatile int *commits_s = abort_s + 1;            // MMA commits issued (thread 0)
  volatile int *issued_s = abort_s + 2;             // TMA chunks issued (thread 0)

  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int v0 = blockIdx.x * kBN, b0 = blockIdx.y * kBM;
  const int nch = (a.K + kKC - 1) / kKC;
  const int segs = nch < kSegs ? nch : kSegs;
  const uint32_t raw_full0 = smem_u32(bars), mma_done0 = smem_u32(bars + kRaw);

  if (tid == 0) {
    for (int i = 0; i < kRaw + kOps; ++i) mbar_init(smem_u32(bars + i), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    *abort_s = 0;
    *commits_s = 0;
    *issued_s = 0;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(const_cast<uint32_t *>(tmem_slot))),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  auto issue_chunk = [&](int c) {
    const int rs = c % kRaw;
    const uint32_t bar = raw_full0 + 8 * rs, dst = smem_u32(raw + rs * kRawBytes);
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(kRawBytes) : "memory");
    tma_load_2d(dst, &tm_h, c * kKC, b0, bar);
    tma_load_2d(dst + kTileA, &tm_w, c * kKC, v0, bar);
  };
  if (tid == 0) {
    const int first = nch < kRaw ? nch : kRaw;
    for (int c = 0; c < first; ++c) issue_chunk(c);
    *issued_s = first;
  }

  bool aborted = false;
  int seg_prev = -1;
  for (int c = 0; c < nch; ++c) {
    const int rs = c % kRaw, os = c % kOps;
    uint8_t *op = ops + os * kOpBytes;
    if (!aborted) {
      bool ok = mbar_wait(raw_full0 + 8 * rs, (c / kRaw) & 1);
      if (ok && c >= kOps) ok = mbar_wait(mma_done0 + 8 * os, ((c - kOps) / kOps) & 1);
      if (ok) {
        const uint8_t *src = raw + rs * kRawBytes;
        split_tile(reinterpret_cast<const float4 *>(src), reinterpret_cast<float4 *>(op),
                   reinterpret_cast<float4 *>(op + kTileA), kTileA / 16, tid);
        split_tile(reinterpret_cast<const float4 *>(src + kTileA), reinterpret_cast<float4 *>(op + 2 * kTileA),
                   reinterpret_cast<float4 *>(op + 2 * kTileA + kTileB), kTileB / 16, tid);
      } else {
        *abort_s = 1;
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    aborted = *abort_s != 0;
    const int seg = c * segs / nch;
    const bool first = seg != seg_prev;
    seg_prev = seg;
    if (aborted || tid != 0) continue;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t a_hi = smem_u32(op), a_lo = a_hi + kTileA, w_hi = a_hi + 2 * kTileA, w_lo = w_hi + kTileB;
    const uint32_t d_main = tmem + seg * kBN, d_corr = tmem + (kSegs + seg) * kBN;
#pragma unroll
    for (int j = 0; j < kKC / 8; ++j) {
      const uint32_t acc = (first && j == 0) ? 0u : 1u, off = j * 32; // 8 tf32 = 32 bytes along k
      mma_tf32(d_main, sw128_desc(a_hi + off), sw128_desc(w_hi + off), acc);
      mma_tf32(d_corr, sw128_desc(a_lo + off), sw128_desc(w_hi + off), acc);
      mma_tf32(d_corr, sw128_desc(a_hi + off), sw128_desc(w_lo + off), 1u);
    }
    mma_commit(mma_done0 + 8 * os);
    *commits_s = c + 1;
    if (c + kRaw < nch) {
      issue_chunk(c + kRaw);
      *issued_s = c + kRaw + 1;
    }
  }
  __syncthreads();
  aborted = *abort_s != 0;
  const int commits = *commits_s, issued = *issued_s;
  bool ready = false;
  if (commits > 0) {
    const int last = commits - 1;
    ready = mbar_wait(mma_done0 + 8 * (last % kOps), (last / kOps) & 1);
  }
  if (aborted && tid == 0) {
    // Bounded wait for TMA chunks still landing in this CTA's shared memory.
    for (int c = commits; c < issued; ++c) mbar_wait(raw_full0 + 8 * (c % kRaw), (c / kRaw) & 1);
  }
  ready = __syncthreads_and(ready) != 0; // the TMEM loads below are warp-collective
  if (aborted || !ready) {
    if (a.err) *reinterpret_cast<volatile int *>(a.err) = 1;
  } else {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const int b = b0 + warp * 32 + lane;
    const uint32_t lane_base = tmem + (uint32_t(warp * 32) << 16);
    float out[32], part[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) out[j] = (a.bias && v0 + j < a.V) ? a.bias[v0 + j] : 0.f;
    for (int s = 0; s < 2 * segs; ++s) {
      const int col = s < segs ? s * kBN : (kSegs + s - segs) * kBN;
      tmem_ld32(lane_base + col, part);
#pragma unroll
      for (int j = 0; j < 32; ++j) out[j] = __fadd_rn(out[j], part[j]);
    }
    if (b < a.B) {
      float *y = a.y + (long)b * a.ldy + v0;
      if (v0 + 32 <= a.V && (a.ldy % 4) == 0 && (reinterpret_cast<uintptr_t>(a.y) & 15) == 0) {
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          *reinterpret_cast<float4 *>(y + j) = make_float4(out[j], out[j + 1], out[j + 2], out[j + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (v0 + j < a.V) y[j] = out[j];
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_tiled() {
  static const EncodeTiled fn = [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<EncodeTiled>(p);
  }();
  return fn;
}

// Row-major fp32 matrix [rows][cols] (row stride ld floats) as TMA boxes of
// kKC columns x box_rows rows, 128-byte swizzle, zero fill out of range.
bool make_map(CUtensorMap *m, const float *p, long rows, long cols, long ld, int box_rows) {
  const EncodeTiled enc = encode_tiled();
  if (!enc) return false;
  const cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(ld) * 4};
  const cuuint32_t box[2] = {cuuint32_t(kKC), cuuint32_t(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(p), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

} // namespace

bool readout_tc_enabled() {
  const char *e = std::getenv("NEUROGEN_READOUT");
  return !(e && std::strcmp(e, "simt") == 0);
}

bool readout_tc_ok(const ReadoutArgs &a) {
  return readout_tc_enabled() && a.B >= 2 && a.K >= 4 && a.K % 4 == 0 && a.ldh % 4 == 0 && a.V >= 1 &&
         aligned16(a.h) && aligned16(a.w) && encode_tiled() != nullptr;
}

void configure_readout_tc() {
  cudaFuncSetAttribute(k_readout_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
}

const void *readout_tc_kernel() { return reinterpret_cast<const void *>(k_readout_tc); }

bool launch_readout_tc(const ReadoutArgs &a, cudaStream_t s) {
  if (!readout_tc_ok(a)) return false;
  CUtensorMap tm_h, tm_w;
  if (!make_map(&tm_h, a.h, a.B, a.K, a.ldh, kBM) || !make_map(&tm_w, a.w, a.V, a.K, a.K, kBN)) return false;
  const dim3 grid((a.V + kBN - 1) / kBN, (a.B + kBM - 1) / kBM);
  k_readout_tc<<<grid, kThreads, kSmemBytes, s>>>(tm_h, tm_w, a);
  return true;
}

} // namespace ngb
