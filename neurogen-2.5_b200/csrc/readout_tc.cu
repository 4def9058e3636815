// Token readout on the 5th-generation tensor cores:
//   logits[b][v] = bias[v] + sum_k h[b][k] * W[v][k]
// (reference: the language model head, neurogen/language/model.py head
// Linear(width, 264), evaluated by the native engine in
// src/native/engine/NeuralEngine.cpp as a sequential fp32 dot product).
//
// The tensor cores read fp32 operands as tf32 (10 explicit mantissa bits), so
// every operand x comes split as hi = x with the low 13 mantissa bits cleared
// (exactly a tf32 value) and lo = x - hi (exact in fp32, read as tf32): the
// head weights once at model load, the hidden state by the LayerNorm kernel
// that produces it.  Then
//   h.W ~= h_hi.W_hi + (h_lo.W_hi + h_hi.W_lo)
// with the small terms in their own TMEM accumulator.  The k range is split
// into up to kSegs segments, one CTA of a kSegs-CTA cluster each; each
// segment's main + correction sum, then the segments' sums, are added in fp32
// in a fixed order, so each accumulator takes few tensor-core additions.  The result is
// within a few 1e-6 of the vector scale of the sequential fp32 sum; it is
// deterministic but not bit-identical to it (the SIMT projection is).
//
// CTA: 128 sessions (TMEM lanes) x 32 vocabulary rows (TMEM columns), 128
// threads.  Thread 0 streams the segment's 32-wide k chunks by TMA
// (SWIZZLE_128B, kStages deep; h hi / lo and W hi / lo per chunk) and issues
// the 12 MMAs of each chunk (4 k-steps x 3 terms, M=128 N=32 K=8), committing
// them to the stage's mbarrier before the stage is refilled.  Each segment
// leaves its sums in its shared memory; after a cluster barrier every CTA adds
// up one slice of the rows over all segments (distributed shared memory) and
// writes those logits.
// Every mbarrier wait is bounded: on a timeout the kernel sets *err, stops
// issuing, waits (bounded) for work in flight, frees its TMEM and returns.
#include "lang_kernels.h"

#include <cooperative_groups.h>
#include <cuda.h>
#include <atomic>
#include <cstdlib>
#include <cstring>

namespace ngb {
namespace {
namespace cg = cooperative_groups;

constexpr int kBM = 128, kBN = 32, kKC = 32;   // sessions, vocab rows, k per chunk
constexpr int kStages = 4, kSegs = 6;          // pipeline stages, k segments (cluster size: 3 clusters fit a GPC)
constexpr int kThreads = 128;
constexpr int kTmemCols = 64;                  // main and correction accumulators of kBN columns
constexpr uint32_t kTileA = kBM * kKC * 4, kTileB = kBN * kKC * 4; // 16 KB, 4 KB
constexpr uint32_t kStageBytes = 2 * (kTileA + kTileB);            // h hi, h lo, W hi, W lo
constexpr int kPartLd = kBN + 4; // row stride of a segment's sums: 16-byte rows, no bank conflict
static_assert(kBM * kPartLd * 4 <= kStages * kStageBytes, "partial sums");
constexpr size_t kSmemBytes = 1024 + kStages * kStageBytes + 256;
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

__global__ void __launch_bounds__(kThreads, 1)
    k_readout_tc(const __grid_constant__ CUtensorMap tm_hh, const __grid_constant__ CUtensorMap tm_hl,
                 const __grid_constant__ CUtensorMap tm_wh, const __grid_constant__ CUtensorMap tm_wl,
                 ReadoutArgs a) {
  extern __shared__ uint8_t smem_raw[];
  // 128-byte swizzled tiles start on 1024-byte boundaries of the shared window.
  uint8_t *stages = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u); // [kStages][hh hl wh wl]
  uint64_t *bars = reinterpret_cast<uint64_t *>(stages + kStages * kStageBytes);   // full[kStages] empty[kStages] done
  volatile uint32_t *tmem_slot = reinterpret_cast<volatile uint32_t *>(bars + 2 * kStages + 1);
  volatile int *abort_s = reinterpret_cast<volatile int *>(tmem_slot + 1);
  // After the MMAs: this segment's sums [row][kPartLd], over the stages.
  float *part = reinterpret_cast<float *>(stages);

  cg::cluster_group cluster = cg::this_cluster();
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int v0 = blockIdx.x * kBN, b0 = blockIdx.y * kBM, z = blockIdx.z; // z: k segment = rank in the cluster
  const int nch = (a.K + kKC - 1) / kKC;
  const int segs = nch < kSegs ? nch : kSegs;
  // Segment z holds the chunks c with c * segs / nch == z.
  const int cb = z < segs ? (z * nch + segs - 1) / segs : nch, ce = z < segs ? ((z + 1) * nch + segs - 1) / segs : nch;
  const int n = ce - cb;
  const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * kStages, done = full0 + 16 * kStages;

  if (tid == 0) {
    for (int i = 0; i < 2 * kStages + 1; ++i) mbar_init(smem_u32(bars + i), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    *abort_s = 0;
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

  if (tid == 0 && n > 0 && a.stall_test) {
    // Test switch: the abort path of a wait that ran out, with nothing in
    // flight yet (no copy or MMA has been issued).
    *abort_s = 1;
  } else if (tid == 0 && n > 0) {
    // Local chunk i (global chunk cb + i) lives in stage i % kStages.
    auto issue_chunk = [&](int i) {
      const int st = i % kStages;
      const uint32_t bar = full0 + 8 * st, dst = smem_u32(stages + st * kStageBytes), k = (cb + i) * kKC;
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(kStageBytes) : "memory");
      tma_load_2d(dst, &tm_hh, k, b0, bar);
      tma_load_2d(dst + kTileA, &tm_hl, k, b0, bar);
      tma_load_2d(dst + 2 * kTileA, &tm_wh, k, v0, bar);
      tma_load_2d(dst + 2 * kTileA + kTileB, &tm_wl, k, v0, bar);
    };
    const int first = n < kStages ? n : kStages;
    for (int i = 0; i < first; ++i) issue_chunk(i);
    int issued = first, consumed = 0, committed = 0;
    bool ok = true;
    for (int i = 0; i < n && ok; ++i) {
      const int st = i % kStages;
      ok = mbar_wait(full0 + 8 * st, (i / kStages) & 1);
      if (!ok) break;
      consumed = i + 1;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t hh = smem_u32(stages + st * kStageBytes), hl = hh + kTileA, wh = hh + 2 * kTileA,
                     wl = wh + kTileB;
#pragma unroll
      for (int j = 0; j < kKC / 8; ++j) {
        const uint32_t acc = (i == 0 && j == 0) ? 0u : 1u, off = j * 32; // 8 tf32 = 32 bytes along k
        mma_tf32(tmem, sw128_desc(hh + off), sw128_desc(wh + off), acc);
        mma_tf32(tmem + kBN, sw128_desc(hl + off), sw128_desc(wh + off), acc);
        mma_tf32(tmem + kBN, sw128_desc(hh + off), sw128_desc(wl + off), 1u);
      }
      mma_commit(empty0 + 8 * st);
      committed = i + 1;
      // Refill the previous chunk's stage once its MMAs have read it.
      const int p = i - 1;
      if (p >= 0 && p + kStages < n) {
        ok = mbar_wait(empty0 + 8 * (p % kStages), (p / kStages) & 1);
        if (ok) issue_chunk(p + kStages), ++issued;
      }
    }
    if (ok) {
      mma_commit(done); // arrives once every MMA above has completed
    } else {
      *abort_s = 1;
      // Bounded waits for the work in flight: the last committed MMAs, then
      // the TMA chunks issued but not consumed.
      if (committed > 0) mbar_wait(empty0 + 8 * ((committed - 1) % kStages), ((committed - 1) / kStages) & 1);
      for (int i = consumed; i < issued; ++i) mbar_wait(full0 + 8 * (i % kStages), (i / kStages) & 1);
    }
  }
  __syncthreads();
  const bool aborted = *abort_s != 0;
  bool ready = n == 0 || (!aborted && mbar_wait(done, 0));
  ready = __syncthreads_and(ready) != 0; // the TMEM loads below are warp-collective
  const bool good = !aborted && ready;
  if (!good && a.err) *reinterpret_cast<volatile int *>(a.err) = 1;
  const int row = warp * 32 + lane;
  float mainv[32] = {}, corrv[32] = {};
  if (good && n > 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t lane_base = tmem + (uint32_t(warp * 32) << 16);
    tmem_ld32(lane_base, mainv);
    tmem_ld32(lane_base + kBN, corrv);
  }
  // The segment's sum (main + correction) of each row, into this CTA's shared memory.
  if (good && n > 0) {
    float4 *dst = reinterpret_cast<float4 *>(part + row * kPartLd);
#pragma unroll
    for (int j = 0; j < kBN; j += 4)
      dst[j / 4] = make_float4(__fadd_rn(mainv[j], corrv[j]), __fadd_rn(mainv[j + 1], corrv[j + 1]),
                               __fadd_rn(mainv[j + 2], corrv[j + 2]), __fadd_rn(mainv[j + 3], corrv[j + 3]));
  }
  cluster.sync(); // every segment's sums are visible cluster-wide
  if (good) {
    // This CTA's slice of the rows: bias, then segments 0..segs-1, a fixed
    // order, read 16 bytes at a time from each segment's shared memory.
    constexpr int kRowsPer = (kBM + kSegs - 1) / kSegs;
    const int r0 = z * kRowsPer, r1 = min(kBM, r0 + kRowsPer);
    for (int it = tid; it < (r1 - r0) * (kBN / 4); it += kThreads) {
      const int r = r0 + it / (kBN / 4), q = it % (kBN / 4), b = b0 + r, v = v0 + 4 * q;
      if (b >= a.B) continue;
      float o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) o[e] = (a.bias && v + e < a.V) ? a.bias[v + e] : 0.f;
      float4 seg[kSegs];
#pragma unroll
      for (int sg = 0; sg < kSegs; ++sg)
        if (sg < segs) seg[sg] = reinterpret_cast<const float4 *>(cluster.map_shared_rank(part, sg) + r * kPartLd)[q];
#pragma unroll
      for (int sg = 0; sg < kSegs; ++sg)
        if (sg < segs) {
          o[0] = __fadd_rn(o[0], seg[sg].x);
          o[1] = __fadd_rn(o[1], seg[sg].y);
          o[2] = __fadd_rn(o[2], seg[sg].z);
          o[3] = __fadd_rn(o[3], seg[sg].w);
        }
      if (a.addv) {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (v + e < a.V) o[e] = __fadd_rn(o[e], __fmul_rn(0.25f, a.addv[(long)b * a.ldadd + v + e]));
      }
      float *y = a.y + (long)b * a.ldy + v;
      if (v + 4 <= a.V && (a.ldy % 4) == 0 && (reinterpret_cast<uintptr_t>(a.y) & 15) == 0) {
        *reinterpret_cast<float4 *>(y) = make_float4(o[0], o[1], o[2], o[3]);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (v + e < a.V) y[e] = o[e];
      }
    }
  }
  cluster.sync(); // every CTA has read the others' sums before any CTA exits
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

// hi = x with the low 13 mantissa bits cleared (a tf32 value), lo = x - hi
// (exact in fp32); the same split k_norm writes for the readout.
__global__ void k_tf32_split(const float *x, const int *xidx, long ldx, int K, float *hi, float *lo) {
  const int b = blockIdx.y, k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= K) return;
  const float v = x[(long)(xidx ? xidx[b] : b) * ldx + k];
  const float h = __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
  hi[(long)b * K + k] = h;
  lo[(long)b * K + k] = __fsub_rn(v, h);
}

} // namespace

void launch_tf32_split(const float *x, const int *xidx, long ldx, int K, int B, float *hi, float *lo,
                       cudaStream_t s) {
  k_tf32_split<<<dim3((K + 255) / 256, B), 256, 0, s>>>(x, xidx, ldx, K, hi, lo);
}

bool projection_tc_enabled() {
  const char *e = std::getenv("NEUROGEN_PROJECTION");
  return e && std::strcmp(e, "tc") == 0;
}

bool readout_tc_enabled() {
  const char *e = std::getenv("NEUROGEN_READOUT");
  return !(e && std::strcmp(e, "simt") == 0);
}

bool readout_tc_ok(const ReadoutArgs &a) {
  return readout_tc_enabled() && a.B >= 2 && a.K >= 4 && a.K % 4 == 0 && a.ldh % 4 == 0 && a.V >= 1 && a.h_hi &&
         a.h_lo && a.w_hi && a.w_lo && aligned16(a.h_hi) && aligned16(a.h_lo) && aligned16(a.w_hi) &&
         aligned16(a.w_lo) && encode_tiled() != nullptr;
}

void configure_readout_tc() {
  cudaFuncSetAttribute(k_readout_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
}

const void *readout_tc_kernel() { return reinterpret_cast<const void *>(k_readout_tc); }

// Test switch NEUROGEN_TEST_READOUT_STALL=k: the first k tensor-core readout
// launches of the process take the kernel's timeout path before issuing any
// copy or MMA, so the error report and the recovery after it can be tested
// without a wait actually running out.
static int take_readout_stall() {
  static std::atomic<int> left{[] {
    const char *e = std::getenv("NEUROGEN_TEST_READOUT_STALL");
    return e ? std::atoi(e) : 0;
  }()};
  int k = left.load();
  while (k > 0 && !left.compare_exchange_weak(k, k - 1)) {
  }
  return k > 0 ? 1 : 0;
}

bool launch_readout_tc(const ReadoutArgs &args, cudaStream_t s) {
  if (!readout_tc_ok(args)) return false;
  ReadoutArgs a = args;
  a.stall_test = take_readout_stall();
  CUtensorMap tm_hh, tm_hl, tm_wh, tm_wl;
  if (!make_map(&tm_hh, a.h_hi, a.B, a.K, a.ldh, kBM) || !make_map(&tm_hl, a.h_lo, a.B, a.K, a.ldh, kBM) ||
      !make_map(&tm_wh, a.w_hi, a.V, a.K, a.K, kBN) || !make_map(&tm_wl, a.w_lo, a.V, a.K, a.K, kBN))
    return false;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.V + kBN - 1) / kBN, (a.B + kBM - 1) / kBM, kSegs);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = kSegs;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, k_readout_tc, tm_hh, tm_hl, tm_wh, tm_wl, a) != cudaSuccess) {
    // A device that cannot place the cluster: clear the launch error; the
    // caller runs the SIMT readout instead.
    (void)cudaGetLastError();
    return false;
  }
  return true;
}

} // namespace ngb
