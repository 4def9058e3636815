// Isolated-tick spiking network: seeded topology generation, CSR / 16x16-block
// layouts by presynaptic neuron, device state and the tick loop.
//
// Generated networks (Erdos-Renyi, fixed fan-in, 16x16 blocks) are deterministic functions of
// the seed through a counter-based generator (splitmix64 of (stream, a, b)),
// so any machine and any thread count produce the same network.  Weights are
// rounded onto the delay ring's fixed-point grid (multiples of 2^-24 nS):
// fp16 weights already are; fp32 weights are rounded once at generation.
#include "net_engine.h"
#include "nccl_dl.h"

#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace ngb {
namespace {

inline uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Independent counter-based streams: value(a, b) for a, b < 2^32.
struct Stream {
  uint64_t key;
  Stream(uint64_t seed, uint64_t id) : key(mix64(seed ^ mix64(id))) {}
  uint64_t bits(uint64_t a, uint64_t b) const { return mix64(((a << 32) | (b & 0xFFFFFFFFull)) ^ key); }
  double uniform(uint64_t a, uint64_t b) const { return double(bits(a, b) >> 11) * 0x1.0p-53; }
  // Uniform integer in [0, m).
  uint64_t below(uint64_t a, uint64_t b, uint64_t m) const {
    return (uint64_t)((unsigned __int128)bits(a, b) * m >> 64);
  }
};

enum : uint64_t { S_EDGE = 1, S_PRE, S_DELAY, S_W1, S_W2, S_BLOCK, S_FILL };

struct WeightDraw {
  const ng_net_config &c;
  Stream w1, w2;
  explicit WeightDraw(const ng_net_config &cfg) : c(cfg), w1(cfg.seed, S_W1), w2(cfg.seed, S_W2) {}
  double normal(uint64_t a, uint64_t b) const {
    const double u1 = (double((w1.bits(a, b) >> 11) + 1)) * 0x1.0p-53; // (0, 1]
    const double u2 = w2.uniform(a, b);
    return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
  }
  // Signed weight keyed by (a, b); inhibitory presynaptic cells are negative.
  // Returns fp32 value and, for fp16 storage, the fp16 bits.
  float draw(uint64_t a, uint64_t b, bool inhibitory, uint16_t *half_bits) const {
    const double z = normal(a, b);
    if (c.weight_kind == NG_W_LOGNORMAL_F32) {
      const double w = std::exp(double(c.w_mu) + double(c.w_sigma) * z);
      float q = float(std::nearbyint(w * 16777216.0) * 0x1.0p-24);
      if (q == 0.f) q = 0x1.0p-24f;
      return inhibitory ? -q : q;
    }
    float m = float(std::fabs(double(c.w_sigma) * z));
    __half h = __float2half_rn(m);
    if (__half2float(h) == 0.f) h = __ushort_as_half(1); // smallest subnormal, 2^-24
    uint16_t bits = __half_as_ushort(h);
    if (inhibitory) bits |= 0x8000u;
    if (half_bits) *half_bits = bits;
    return __half2float(__ushort_as_half(bits));
  }
};

inline uint32_t pack_word(int post, int delay) { return uint32_t(post) | (uint32_t(delay - 1) << 28); }

long long pad8(long long x) { return (x + 7) & ~7LL; }

// Per-postsynaptic-neuron bound on the summed fixed-point input of one slot.
void check_ring_bound(int n, const std::vector<double> &sum_e, const std::vector<double> &sum_i) {
  for (int j = 0; j < n; ++j)
    if (sum_e[j] >= 127.0 || sum_i[j] >= 127.0)
      throw std::invalid_argument("Synaptic input of neuron " + std::to_string(j) +
                                  " can exceed the delay ring's fixed-point range (127 nS per slot)");
}

void finish_rows(HostCSR &out, const std::vector<long long> &count) {
  const int n = out.n;
  out.row.assign(size_t(n) + 1, 0);
  for (int i = 0; i < n; ++i) out.row[i + 1] = out.row[i] + pad8(count[i]);
  const size_t total = size_t(out.row[n]);
  out.syn.assign(total, pack_word(0, 1));
  out.outdeg.assign(n, 0);
}

} // namespace

void validate_config(const ng_net_config &c) {
  if (c.n < 1 || c.n > int(kPostMask)) throw std::invalid_argument("Network size must be in 1..2^28-1");
  if (c.n_exc < 0 || c.n_exc > c.n) throw std::invalid_argument("n_exc must be in 0..n");
  if (c.delay_min < 1 || c.delay_max < c.delay_min || c.delay_max > kRingSlots - 1)
    throw std::invalid_argument("Delays must satisfy 1 <= delay_min <= delay_max <= 15");
  if (c.weight_kind != NG_W_LOGNORMAL_F32 && c.weight_kind != NG_W_HALFNORMAL_F16)
    throw std::invalid_argument("Unknown weight kind");
  if (!(c.dt_ms > 0) || !(c.cap_exc_pf > 0) || !(c.cap_inh_pf > 0) || !(c.g_leak_ns > 0) ||
      !(c.tau_exc_ms > 0) || !(c.tau_inh_ms > 0) || !(c.tau_adapt_ms > 0) || !(c.t_ref_ms >= 0))
    throw std::invalid_argument("Membrane constants must be positive");
  const float vals[] = {c.e_leak_mv, c.e_inh_mv, c.v_thresh_mv, c.v_reset_mv, c.adapt_inc_pa, c.bias_pa,
                        c.drive_p, c.drive_ns, c.p_connect, c.w_mu, c.w_sigma};
  for (float v : vals)
    if (!std::isfinite(v)) throw std::invalid_argument("Network parameters must be finite");
  if (c.drive_kind != NG_DRIVE_CONDUCTANCE && c.drive_kind != NG_DRIVE_IMPOSED)
    throw std::invalid_argument("Unknown drive kind");
  if (c.drive_p < 0 || c.drive_p > 1) throw std::invalid_argument("drive_p must be in [0, 1]");
  if (c.storage != 0 && c.storage != 1) throw std::invalid_argument("storage must be 0 (CSR) or 1 (BSR)");
  if (c.launch < 0 || c.launch > 3)
    throw std::invalid_argument("launch must be 0 (auto), 1 (fused), 2 (split) or 3 (resident)");
  if (c.launch == 3 && c.part_world > 1)
    throw std::invalid_argument("The resident launch needs an unpartitioned network");
  if (c.plasticity != 0 && c.plasticity != 1) throw std::invalid_argument("plasticity must be 0 or 1");
  if (c.plasticity) {
    if (!(c.stdp_rate >= 0) || !(c.inhibitory_rate >= 0) || !std::isfinite(c.stdp_rate) ||
        !std::isfinite(c.inhibitory_rate) || !(c.target_hz > 0) || !std::isfinite(c.target_hz) ||
        !(c.scaling_tau_ms > 0) || !std::isfinite(c.scaling_tau_ms))
      throw std::invalid_argument("Learning rates must be finite and nonnegative, target_hz and scaling_tau_ms positive");
    if (c.part_world > 1 || c.storage != 0 || c.weight_kind != NG_W_LOGNORMAL_F32 || c.launch == 1 || c.launch == 3)
      throw std::invalid_argument("Learning needs fp32 weights, CSR storage, an unpartitioned network and the split launch");
  }
  switch (c.topology) {
  case NG_TOPO_ERDOS_RENYI:
    if (!(c.p_connect >= 0 && c.p_connect <= 1)) throw std::invalid_argument("p_connect must be in [0, 1]");
    break;
  case NG_TOPO_FIXED_FANIN:
    if (c.fanin < 0 || c.n < 2) throw std::invalid_argument("fixed fan-in needs fanin >= 0 and n >= 2");
    break;
  case NG_TOPO_BSR16:
    if (c.n % 16) throw std::invalid_argument("16x16 block topology needs n divisible by 16");
    if (c.bsr_blocks < 0 || c.bsr_blocks > c.n / 16) throw std::invalid_argument("bsr_blocks out of range");
    if (c.bsr_fill < 1 || c.bsr_fill > 256) throw std::invalid_argument("bsr_fill must be in 1..256");
    if (c.weight_kind != NG_W_HALFNORMAL_F16) throw std::invalid_argument("16x16 blocks store fp16 weights");
    break;
  default:
    throw std::invalid_argument("Unknown topology");
  }
  if (c.storage == 1 && c.topology != NG_TOPO_BSR16)
    throw std::invalid_argument("Block storage needs the 16x16 block topology");
  if (c.part_world < 0 || c.part_world > 1024) throw std::invalid_argument("part_world must be in 0..1024");
  if (c.part_world > 1) {
    if (c.part_rank < 0 || c.part_rank >= c.part_world) throw std::invalid_argument("part_rank must be in 0..part_world-1");
    if (c.n % (32 * c.part_world)) throw std::invalid_argument("A partitioned network needs n divisible by 32 * part_world");
    if (c.storage != 0 || c.topology == NG_TOPO_BSR16)
      throw std::invalid_argument("A partitioned network uses CSR storage with Erdos-Renyi or fixed fan-in topology");
  }
}

// ---------------------------------------------------------------------------
// CSR generation.
// ---------------------------------------------------------------------------
// Postsynaptic range [lo, hi) held by this partition (the whole network when
// unpartitioned).
static void partition_range(const ng_net_config &c, int &lo, int &hi) {
  const int world = c.part_world > 1 ? c.part_world : 1;
  const int rank = c.part_world > 1 ? c.part_rank : 0;
  lo = int((long long)c.n * rank / world);
  hi = int((long long)c.n * (rank + 1) / world);
}

void generate_csr(const ng_net_config &c, HostCSR &out) {
  const int n = c.n;
  int lo = 0, hi = n;
  partition_range(c, lo, hi);
  const int np = hi - lo;
  out.n = n;
  out.post_base = lo;
  out.n_post = np;
  const WeightDraw wd(c);
  const Stream edge(c.seed, S_EDGE), pres(c.seed, S_PRE), dly(c.seed, S_DELAY);
  const uint64_t dspan = uint64_t(c.delay_max - c.delay_min + 1);
  const bool half = c.weight_kind == NG_W_HALFNORMAL_F16;
  std::vector<double> sum_e(np, 0.0), sum_i(np, 0.0);

  if (c.topology == NG_TOPO_ERDOS_RENYI) {
    // Row by row (presynaptic), held posts in ascending order.
    std::vector<long long> count(n, 0);
#pragma omp parallel for schedule(dynamic, 64)
    for (int i = 0; i < n; ++i) {
      long long k = 0;
      for (int j = lo; j < hi; ++j)
        if (j != i && edge.uniform(uint64_t(i), uint64_t(j)) < double(c.p_connect)) ++k;
      count[i] = k;
    }
    finish_rows(out, count);
    if (half) out.w16.assign(out.syn.size(), 0);
    else out.w32.assign(out.syn.size(), 0.f);
#pragma omp parallel for schedule(dynamic, 64)
    for (int i = 0; i < n; ++i) {
      long long e = out.row[i];
      const bool inh = i >= c.n_exc;
      for (int j = lo; j < hi; ++j) {
        if (j == i || !(edge.uniform(uint64_t(i), uint64_t(j)) < double(c.p_connect))) continue;
        const int d = c.delay_min + int(dly.below(uint64_t(i), uint64_t(j), dspan));
        out.syn[e] = pack_word(j - lo, d);
        uint16_t hb = 0;
        const float w = wd.draw(uint64_t(i), uint64_t(j), inh, &hb);
        if (half) out.w16[e] = hb;
        else out.w32[e] = w;
        ++e;
      }
      out.outdeg[i] = int(count[i]);
    }
    for (int i = 0; i < n; ++i)
      for (long long e = out.row[i]; e < out.row[i] + out.outdeg[i]; ++e) {
        const double w = half ? double(__half2float(__ushort_as_half(out.w16[e]))) : double(out.w32[e]);
        (w < 0 ? sum_i : sum_e)[out.syn[e] & kPostMask] += std::fabs(w);
      }
  } else if (c.topology == NG_TOPO_FIXED_FANIN) {
    // Each held post j draws `fanin` uniform presynaptic cells keyed (j, k) (no
    // autapse: a draw of j itself moves to the next cell).  Two passes over a
    // fixed split of the posts into kChunks: count per (chunk, pre), then each
    // chunk writes its synapses in post order at its own offsets -- rows come
    // out in ascending post order whatever the thread count, without holding
    // every synapse twice.
    const int K = c.fanin;
    constexpr int kChunks = 8;
    auto chunk_lo = [&](int ch) { return lo + int((long long)np * ch / kChunks); };
    auto draw_pre = [&](int j, int k) {
      int pre = int(pres.below(uint64_t(j), uint64_t(k), uint64_t(n)));
      return pre == j ? (pre + 1) % n : pre;
    };
    std::vector<int> cnt(size_t(kChunks) * n, 0);
#pragma omp parallel for schedule(dynamic, 1)
    for (int ch = 0; ch < kChunks; ++ch) {
      int *cc = cnt.data() + size_t(ch) * n;
      for (int j = chunk_lo(ch); j < chunk_lo(ch + 1); ++j)
        for (int k = 0; k < K; ++k) ++cc[draw_pre(j, k)];
    }
    std::vector<long long> count(n, 0);
    for (int ch = 0; ch < kChunks; ++ch)
      for (int i = 0; i < n; ++i) count[i] += cnt[size_t(ch) * n + i];
    finish_rows(out, count);
    if (half) out.w16.assign(out.syn.size(), 0);
    else out.w32.assign(out.syn.size(), 0.f);
    // cursor[ch][pre]: where chunk ch writes its first synapse of row pre.
    std::vector<long long> cursor(size_t(kChunks) * n);
    for (int i = 0; i < n; ++i) {
      long long at = out.row[i];
      for (int ch = 0; ch < kChunks; ++ch) {
        cursor[size_t(ch) * n + i] = at;
        at += cnt[size_t(ch) * n + i];
      }
    }
#pragma omp parallel for schedule(dynamic, 1)
    for (int ch = 0; ch < kChunks; ++ch) {
      long long *cur = cursor.data() + size_t(ch) * n;
      for (int j = chunk_lo(ch); j < chunk_lo(ch + 1); ++j)
        for (int k = 0; k < K; ++k) {
          const int pre = draw_pre(j, k);
          const long long e = cur[pre]++;
          out.syn[e] = pack_word(j - lo, c.delay_min + int(dly.below(uint64_t(j), uint64_t(k), dspan)));
          uint16_t hb = 0;
          const float w = wd.draw(uint64_t(j), uint64_t(k), pre >= c.n_exc, &hb);
          if (half) out.w16[e] = hb;
          else out.w32[e] = w;
          const double wa = half ? double(__half2float(__ushort_as_half(hb))) : double(w);
          (wa < 0 ? sum_i : sum_e)[j - lo] += std::fabs(wa); // post j belongs to this chunk only
        }
    }
    for (int i = 0; i < n; ++i) out.outdeg[i] = int(count[i]);
  } else {
    // 16x16 block topology stored as CSR (same matrix as the block storage).
    HostBSR b;
    generate_bsr(c, b);
    std::vector<long long> count(n, 0);
    for (int i = 0; i < n; ++i) count[i] = b.outdeg[i];
    finish_rows(out, count);
    out.w16.assign(out.syn.size(), 0);
    for (int bc = 0; bc < b.nb; ++bc)
      for (int col = 0; col < 16; ++col) {
        const int pre = bc * 16 + col;
        long long e = out.row[pre];
        for (long long k = b.bcol[bc]; k < b.bcol[bc + 1]; ++k) {
          const int br = int(b.blk[k] & kPostMask);
          const int d = int(b.blk[k] >> 28) + 1;
          for (int r = 0; r < 16; ++r) {
            const uint16_t hb = b.tiles[(size_t(k) * 16 + col) * 16 + r];
            if ((hb & 0x7FFFu) == 0) continue;
            out.syn[e] = pack_word(br * 16 + r, d);
            out.w16[e] = hb;
            ++e;
            const double w = double(__half2float(__ushort_as_half(hb)));
            (w < 0 ? sum_i : sum_e)[br * 16 + r] += std::fabs(w);
          }
        }
        out.outdeg[pre] = int(count[pre]);
      }
  }
  check_ring_bound(np, sum_e, sum_i);
}

// ---------------------------------------------------------------------------
// 16x16 block generation: per block-row, `bsr_blocks` distinct block-columns
// and, per block, `bsr_fill` distinct entries (Floyd's sampling), one delay
// per block.  Stored by block-column, blocks in ascending block-row order.
// ---------------------------------------------------------------------------
namespace {
// Floyd's algorithm: m distinct values of [0, range), keyed draws (a, salt+j).
void floyd(const Stream &s, uint64_t a, uint64_t salt, int range, int m, std::vector<int> &out) {
  out.clear();
  for (int j = range - m; j < range; ++j) {
    const int t = int(s.below(a, salt + uint64_t(j), uint64_t(j) + 1));
    if (std::find(out.begin(), out.end(), t) == out.end()) out.push_back(t);
    else out.push_back(j);
  }
  std::sort(out.begin(), out.end());
}
} // namespace

void generate_bsr(const ng_net_config &c, HostBSR &out) {
  const int n = c.n, NB = n / 16, M = c.bsr_blocks, F = c.bsr_fill;
  out.nb = NB;
  const WeightDraw wd(c);
  const Stream blk(c.seed, S_BLOCK), fill(c.seed, S_FILL), dly(c.seed, S_DELAY);
  const uint64_t dspan = uint64_t(c.delay_max - c.delay_min + 1);
  // By block-row first.
  std::vector<int> rcols(size_t(NB) * M);
  std::vector<uint32_t> rmeta(size_t(NB) * M);
  std::vector<uint16_t> rtiles(size_t(NB) * M * 256, 0);
#pragma omp parallel
  {
    std::vector<int> cols, pos;
#pragma omp for schedule(dynamic, 16)
    for (int br = 0; br < NB; ++br) {
      floyd(blk, uint64_t(br), 0, NB, M, cols);
      for (int m = 0; m < M; ++m) {
        const int bc = cols[m];
        const size_t x = size_t(br) * M + m;
        rcols[x] = bc;
        rmeta[x] = pack_word(br, c.delay_min + int(dly.below(uint64_t(br), uint64_t(bc), dspan)));
        floyd(fill, uint64_t(br), uint64_t(bc) * 256, 256, F, pos);
        for (int p : pos) {
          const int r = p / 16, col = p % 16; // entry (post row r, pre column col)
          const int pre = bc * 16 + col;
          uint16_t hb = 0;
          wd.draw(uint64_t(br) * 16 + r, uint64_t(pre), pre >= c.n_exc, &hb);
          rtiles[x * 256 + size_t(col) * 16 + r] = hb;
        }
      }
    }
  }
  // Regroup by block-column (stable in block-row order).
  out.bcol.assign(size_t(NB) + 1, 0);
  for (size_t x = 0; x < rcols.size(); ++x) out.bcol[rcols[x] + 1]++;
  for (int b = 0; b < NB; ++b) out.bcol[b + 1] += out.bcol[b];
  const size_t nblk = rcols.size();
  out.blk.assign(nblk, 0);
  out.tiles.assign(nblk * 256, 0);
  std::vector<long long> at(out.bcol.begin(), out.bcol.end() - 1);
  std::vector<double> sum_e(n, 0.0), sum_i(n, 0.0);
  out.outdeg.assign(n, 0);
  for (size_t x = 0; x < nblk; ++x) {
    const long long k = at[rcols[x]]++;
    out.blk[k] = rmeta[x];
    std::memcpy(&out.tiles[size_t(k) * 256], &rtiles[x * 256], 512);
    const int br = int(rmeta[x] & kPostMask), bc = rcols[x];
    for (int col = 0; col < 16; ++col)
      for (int r = 0; r < 16; ++r) {
        const uint16_t hb = rtiles[x * 256 + size_t(col) * 16 + r];
        if ((hb & 0x7FFFu) == 0) continue;
        out.outdeg[bc * 16 + col]++;
        const double w = double(__half2float(__ushort_as_half(hb)));
        (w < 0 ? sum_i : sum_e)[br * 16 + r] += std::fabs(w);
      }
  }
  check_ring_bound(n, sum_e, sum_i);
}

void csr_from_edges(const ng_net_config &c, int64_t nnz, const int32_t *pre, const int32_t *post,
                    const int32_t *delay, const float *w, HostCSR &out) {
  const int n = c.n;
  out.n = n;
  out.post_base = 0;
  out.n_post = n;
  if (nnz < 0 || (nnz > 0 && (!pre || !post || !delay || !w)))
    throw std::invalid_argument("Null synapse arrays");
  std::vector<long long> count(n, 0);
  std::vector<double> sum_e(n, 0.0), sum_i(n, 0.0);
  for (int64_t e = 0; e < nnz; ++e) {
    if (pre[e] < 0 || pre[e] >= n || post[e] < 0 || post[e] >= n)
      throw std::invalid_argument("Synapse endpoint out of range");
    if (delay[e] < 1 || delay[e] > kRingSlots - 1) throw std::invalid_argument("Synapse delay must be in 1..15");
    if (!std::isfinite(w[e])) throw std::invalid_argument("Non-finite synaptic weight");
    const double q = double(std::fabs(w[e])) * 16777216.0;
    if (q != std::floor(q)) throw std::invalid_argument("Weights must be multiples of 2^-24 nS");
    if (w[e] == 0.f) continue;
    ++count[pre[e]];
    (w[e] < 0 ? sum_i : sum_e)[post[e]] += std::fabs(double(w[e]));
  }
  check_ring_bound(n, sum_e, sum_i);
  finish_rows(out, count);
  out.w32.assign(out.syn.size(), 0.f);
  std::vector<long long> fill(out.row.begin(), out.row.end() - 1);
  for (int64_t e = 0; e < nnz; ++e) {
    if (w[e] == 0.f) continue;
    const long long k = fill[pre[e]]++;
    out.syn[k] = pack_word(post[e], delay[e]);
    out.w32[k] = w[e];
  }
  for (int i = 0; i < n; ++i) out.outdeg[i] = int(count[i]);
}

// ---------------------------------------------------------------------------
// Delay split: the synapses whose delivery the next tick waits for (delay 1)
// go first in every row, so that the rest can be pushed while the next tick
// already runs.  Stable within each segment.
// ---------------------------------------------------------------------------
void split_by_delay(HostCSR &h) {
  const int n = h.n;
  const bool half = !h.w16.empty();
  std::vector<int> d1(n, 0);
#pragma omp parallel for schedule(static)
  for (int i = 0; i < n; ++i) {
    int c1 = 0;
    for (long long e = h.row[i]; e < h.row[i] + h.outdeg[i]; ++e) c1 += (h.syn[e] >> 28) == 0;
    d1[i] = c1;
  }
  std::vector<long long> row(size_t(n) + 1, 0);
  h.mid.assign(n, 0);
  for (int i = 0; i < n; ++i) {
    h.mid[i] = int(pad8(d1[i]));
    row[i + 1] = row[i] + pad8(d1[i]) + pad8(h.outdeg[i] - d1[i]);
  }
  const size_t total = size_t(row[n]);
  std::vector<uint32_t> syn(total, pack_word(0, 1));
  std::vector<uint16_t> w16(half ? total : 0, 0);
  std::vector<float> w32(half ? 0 : total, 0.f);
#pragma omp parallel for schedule(static)
  for (int i = 0; i < n; ++i) {
    long long a = row[i], b = row[i] + h.mid[i];
    for (long long e = h.row[i]; e < h.row[i] + h.outdeg[i]; ++e) {
      const long long to = (h.syn[e] >> 28) == 0 ? a++ : b++;
      syn[to] = h.syn[e];
      if (half) w16[to] = h.w16[e];
      else w32[to] = h.w32[e];
    }
  }
  h.row.swap(row);
  h.syn.swap(syn);
  if (half) h.w16.swap(w16);
  else h.w32.swap(w32);
}

void split_by_delay(HostBSR &b) {
  b.mid.assign(b.nb, 0);
#pragma omp parallel for schedule(static)
  for (int bc = 0; bc < b.nb; ++bc) {
    const long long b0 = b.bcol[bc], b1 = b.bcol[bc + 1];
    std::vector<uint32_t> meta(b.blk.begin() + b0, b.blk.begin() + b1);
    std::vector<uint16_t> tiles(b.tiles.begin() + b0 * 256, b.tiles.begin() + b1 * 256);
    long long at = b0;
    for (int pass = 0; pass < 2; ++pass)
      for (long long k = 0; k < b1 - b0; ++k) {
        const bool first = (meta[k] >> 28) == 0;
        if (first != (pass == 0)) continue;
        b.blk[at] = meta[k];
        std::copy(tiles.begin() + k * 256, tiles.begin() + (k + 1) * 256, b.tiles.begin() + at * 256);
        ++at;
      }
    int ones = 0;
    for (uint32_t m : meta) ones += (m >> 28) == 0;
    b.mid[bc] = ones;
  }
}

// ---------------------------------------------------------------------------
// Host topology objects.
// ---------------------------------------------------------------------------
int64_t Topology::synapses() const {
  int64_t total = 0;
  for (int x : blocks ? bsr.outdeg : csr.outdeg) total += x;
  return total;
}

void Topology::export_edges(int32_t *pre, int32_t *post, int32_t *delay, float *weight) const {
  size_t k = 0;
  auto emit = [&](int p, int q, int d, float w) {
    if (pre) pre[k] = p;
    if (post) post[k] = q;
    if (delay) delay[k] = d;
    if (weight) weight[k] = w;
    ++k;
  };
  if (blocks) {
    for (int bc = 0; bc < bsr.nb; ++bc)
      for (int col = 0; col < 16; ++col)
        for (long long b = bsr.bcol[bc]; b < bsr.bcol[bc + 1]; ++b) {
          const int br = int(bsr.blk[b] & kPostMask), d = int(bsr.blk[b] >> 28) + 1;
          for (int r = 0; r < 16; ++r) {
            const uint16_t hb = bsr.tiles[(size_t(b) * 16 + col) * 16 + r];
            if ((hb & 0x7FFFu) == 0) continue;
            emit(bc * 16 + col, br * 16 + r, d, __half2float(__ushort_as_half(hb)));
          }
        }
    return;
  }
  const bool half = !csr.w16.empty();
  for (int i = 0; i < csr.n; ++i)
    for (long long e = csr.row[i]; e < csr.row[i + 1]; ++e) {
      const float w = half ? __half2float(__ushort_as_half(csr.w16[e])) : csr.w32[e];
      if (w != 0.f) emit(i, csr.post_base + int(csr.syn[e] & kPostMask), int(csr.syn[e] >> 28) + 1, w);
    }
}

Topology *make_topology(const ng_net_config &cfg) {
  validate_config(cfg);
  auto t = std::make_unique<Topology>();
  t->cfg = cfg;
  t->blocks = cfg.storage == 1;
  if (t->blocks) {
    generate_bsr(cfg, t->bsr);
    split_by_delay(t->bsr);
  } else {
    generate_csr(cfg, t->csr);
    split_by_delay(t->csr);
  }
  return t.release();
}

Topology *make_topology_edges(const ng_net_config &cfg, int64_t nnz, const int32_t *pre, const int32_t *post,
                              const int32_t *delay, const float *w) {
  ng_net_config c = cfg;
  c.storage = 0;
  c.topology = NG_TOPO_ERDOS_RENYI; // topology fields are unused for explicit edges
  c.p_connect = 0.f;
  c.weight_kind = NG_W_LOGNORMAL_F32;
  validate_config(c);
  auto t = std::make_unique<Topology>();
  t->cfg = c;
  csr_from_edges(c, nnz, pre, post, delay, w, t->csr);
  split_by_delay(t->csr);
  return t.release();
}

// ---------------------------------------------------------------------------
// Device network.
// ---------------------------------------------------------------------------
namespace {
template <class T> DeviceBuffer upload_vec(const std::vector<T> &v) {
  DeviceBuffer d(std::max<size_t>(v.size(), 1) * sizeof(T));
  if (!v.empty()) NGB_CUDA(cudaMemcpy(d.as<void>(), v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice));
  return d;
}
// Upload with `pad` zero elements after the data (vector loads may read past a row end).
template <class T> DeviceBuffer upload_padded(const std::vector<T> &v, size_t pad) {
  DeviceBuffer d((v.size() + pad) * sizeof(T));
  NGB_CUDA(cudaMemset(d.as<void>(), 0, (v.size() + pad) * sizeof(T)));
  if (!v.empty()) NGB_CUDA(cudaMemcpy(d.as<void>(), v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice));
  return d;
}
float decay_of(float dt, float tau) { return float(std::exp(-double(dt) / double(tau))); }
} // namespace

Network::Network(const Topology &topo, const void *nccl_id) : cfg(topo.cfg) {
  const ng_net_config &c = topo.cfg;
  const HostCSR *csr = topo.blocks ? nullptr : &topo.csr;
  const HostBSR *bsr = topo.blocks ? &topo.bsr : nullptr;
  device = require_sm100_device();
  // Held neurons [base, base + n_) of a network of n_pre_ neurons.
  n_pre_ = c.n;
  n_ = csr ? csr->n_post : c.n;
  base_ = csr ? csr->post_base : 0;
  world_ = c.part_world > 1 ? c.part_world : 1;
  rank_ = world_ > 1 ? c.part_rank : 0;
  NetDev &d = dev_;
  d.n = n_;
  d.n_exc = c.n_exc;
  d.n_pre = n_pre_;
  d.base = base_;
  if (bsr) {
    bcol_ = upload_vec(bsr->bcol);
    blk_ = upload_vec(bsr->blk);
    tiles_ = upload_vec(bsr->tiles);
    outdeg_ = upload_vec(bsr->outdeg);
    if (int(bsr->mid.size()) != bsr->nb) throw std::logic_error("block-columns not split by delay");
    mid_ = upload_vec(bsr->mid);
    d.bsr = 1;
    d.bcol = bcol_.as<long long>();
    d.blk = blk_.as<uint32_t>();
    d.tiles = tiles_.as<uint16_t>();
    d.bmid = mid_.as<int>();
    for (int x : bsr->outdeg) nnz_ += x;
  } else {
    row_ = upload_vec(csr->row);
    syn_ = upload_padded(csr->syn, kTailPad);
    outdeg_ = upload_vec(csr->outdeg);
    if (!csr->w16.empty() || csr->w32.empty()) {
      w_ = upload_padded(csr->w16.empty() ? std::vector<uint16_t>(csr->syn.size(), 0) : csr->w16, kTailPad);
      d.w_half = 1;
    } else {
      w_ = upload_padded(csr->w32, kTailPad);
      d.w_half = 0;
    }
    if (int(csr->mid.size()) != csr->n) throw std::logic_error("CSR rows not split by delay");
    mid_ = upload_vec(csr->mid);
    d.row = row_.as<long long>();
    d.syn = syn_.as<uint32_t>();
    d.w = w_.as<void>();
    d.mid = mid_.as<int>();
    for (int x : csr->outdeg) nnz_ += x;
  }
  int max_delay = 1;
  for (uint32_t w : csr ? csr->syn : bsr->blk) max_delay = std::max(max_delay, int(w >> 28) + 1);
  init_state(nccl_id, max_delay);
}

// Partitioned fixed fan-in network whose synapses are drawn on the device:
// the rank holds posts [lo, hi) and the rows of every presynaptic cell onto them.
Network::Network(const ng_net_config &c, const void *nccl_id, DeviceFanin) : cfg(c) {
  validate_config(c);
  if (c.topology != NG_TOPO_FIXED_FANIN || c.storage != 0 || c.weight_kind != NG_W_HALFNORMAL_F16)
    throw std::invalid_argument("Device generation covers fixed fan-in CSR networks with fp16 weights");
  device = require_sm100_device();
  int lo = 0, hi = 0;
  partition_range(c, lo, hi);
  n_pre_ = c.n;
  n_ = hi - lo;
  base_ = lo;
  world_ = c.part_world > 1 ? c.part_world : 1;
  rank_ = world_ > 1 ? c.part_rank : 0;
  NetDev &d = dev_;
  d.n = n_;
  d.n_exc = c.n_exc;
  d.n_pre = n_pre_;
  d.base = base_;
  generate_fanin_device(lo, hi);
  init_state(nccl_id, c.delay_max);
}

void Network::generate_fanin_device(int lo, int hi) {
  const ng_net_config &c = cfg;
  const int n = c.n;
  FaninGen g{};
  g.n = n;
  g.n_exc = c.n_exc;
  g.lo = lo;
  g.np = hi - lo;
  g.fanin = c.fanin;
  g.delay_min = c.delay_min;
  g.delay_span = c.delay_max - c.delay_min + 1;
  g.sigma = c.w_sigma;
  g.key_pre = Stream(c.seed, S_PRE).key;
  g.key_delay = Stream(c.seed, S_DELAY).key;
  g.key_w1 = Stream(c.seed, S_W1).key;
  g.key_w2 = Stream(c.seed, S_W2).key;
  // Pass 1: synapses per row, delay-1 apart -> padded row layout on the host.
  DeviceBuffer c12(size_t(n) * 8 + 4);
  int *c1 = c12.as<int>(), *c2 = c1 + n, *bad = c2 + n;
  NGB_CUDA(cudaMemset(c1, 0, size_t(n) * 8));
  NGB_CUDA(cudaMemset(bad, 0x7F, 4));
  launch_fanin_count(g, c1, c2, nullptr);
  NGB_CUDA(cudaGetLastError());
  std::vector<int> h1(n), h2(n), mid(n), outdeg(n);
  NGB_CUDA(cudaMemcpy(h1.data(), c1, size_t(n) * 4, cudaMemcpyDeviceToHost));
  NGB_CUDA(cudaMemcpy(h2.data(), c2, size_t(n) * 4, cudaMemcpyDeviceToHost));
  std::vector<long long> row(size_t(n) + 1, 0);
  for (int i = 0; i < n; ++i) {
    mid[i] = int(pad8(h1[i]));
    outdeg[i] = h1[i] + h2[i];
    nnz_ += outdeg[i];
    row[i + 1] = row[i] + pad8(h1[i]) + pad8(h2[i]);
  }
  const size_t total = size_t(row[n]) + kTailPad;
  row_ = upload_vec(row);
  mid_ = upload_vec(mid);
  outdeg_ = upload_vec(outdeg);
  syn_.reset(total * 4);
  w_.reset(total * 2);
  NGB_CUDA(cudaMemset(syn_.as<void>(), 0, total * 4)); // padding: post 0, delay 1, weight 0
  NGB_CUDA(cudaMemset(w_.as<void>(), 0, total * 2));
  // Pass 2: place the synapses (the counters become cursors).
  NGB_CUDA(cudaMemset(c1, 0, size_t(n) * 8));
  launch_fanin_fill(g, row_.as<long long>(), mid_.as<int>(), c1, c2, syn_.as<uint32_t>(), w_.as<uint16_t>(), bad,
                    nullptr);
  NGB_CUDA(cudaGetLastError());
  int bad_post = 0;
  NGB_CUDA(cudaMemcpy(&bad_post, bad, 4, cudaMemcpyDeviceToHost));
  if (bad_post != 0x7F7F7F7F)
    throw std::invalid_argument("Synaptic input of neuron " + std::to_string(bad_post) +
                                " can exceed the delay ring's fixed-point range (127 nS per slot)");
  NetDev &d = dev_;
  d.row = row_.as<long long>();
  d.syn = syn_.as<uint32_t>();
  d.w = w_.as<void>();
  d.w_half = 1;
  d.mid = mid_.as<int>();
}

// State, counters, launch shape and (partitioned) communicator; the synapses
// are on the device already.
void Network::init_state(const void *nccl_id, int max_delay) {
  const ng_net_config &c = cfg;
  NetDev &d = dev_;
  d.outdeg = outdeg_.as<int>();
  const size_t N = size_t(n_);
  v_.reset(N * 4);
  a_.reset(N * 4);
  ge_.reset(N * 4);
  gi_.reset(N * 4);
  ref_.reset(N * 4);
  ring_.reset(size_t(kRingSlots) * N * 8);
  std::vector<float> v0(N, c.e_leak_mv);
  NGB_CUDA(cudaMemcpy(v_.as<float>(), v0.data(), N * 4, cudaMemcpyHostToDevice));
  NGB_CUDA(cudaMemset(a_.as<float>(), 0, N * 4));
  NGB_CUDA(cudaMemset(ge_.as<float>(), 0, N * 4));
  NGB_CUDA(cudaMemset(gi_.as<float>(), 0, N * 4));
  NGB_CUDA(cudaMemset(ref_.as<int>(), 0, N * 4));
  NGB_CUDA(cudaMemset(ring_.as<int2>(), 0, size_t(kRingSlots) * N * 8));
  d.v = v_.as<float>();
  d.a = a_.as<float>();
  d.ge = ge_.as<float>();
  d.gi = gi_.as<float>();
  d.ref = ref_.as<int>();
  d.ring = ring_.as<int2>();
  d.dE = decay_of(c.dt_ms, c.tau_exc_ms);
  d.dI = decay_of(c.dt_ms, c.tau_inh_ms);
  d.dA = decay_of(c.dt_ms, c.tau_adapt_ms);
  d.g_leak = c.g_leak_ns;
  d.gLEL = c.g_leak_ns * c.e_leak_mv;
  d.e_inh = c.e_inh_mv;
  d.v_th = c.v_thresh_mv;
  d.v_reset = c.v_reset_mv;
  d.cap_e = c.cap_exc_pf;
  d.cap_i = c.cap_inh_pf;
  d.neg_dt = -c.dt_ms;
  d.adapt_inc = c.adapt_inc_pa;
  d.bias = c.bias_pa;
  d.drive_ns = c.drive_ns;
  d.drive_kind = c.drive_kind;
  const double thr = double(c.drive_p) * 4294967296.0;
  d.drive_thr = thr >= 4294967295.0 ? 0xFFFFFFFFu : uint32_t(thr);
  d.drive_key = mix64(c.seed ^ 0xD41Eull);
  d.ref_ticks = int(std::lround(double(c.t_ref_ms) / double(c.dt_ms)));
  // Whole-network bitmask (padded to whole 256-neuron groups) twice, for
  // even and odd ticks; per-group counters (enough for the held groups and
  // the presynaptic groups); tick.
  // Resident launch (persistent kernel, state in shared memory) when asked
  // for, or by default when the network qualifies and fits.
  if (world_ == 1 && !c.plasticity && (c.launch == 3 || c.launch == 0))
    resident_ = plan_resident(max_delay, c.launch == 3);
  const size_t pre_groups = (size_t(n_pre_) + kNetBlock - 1) / kNetBlock;
  const size_t groups = std::max({pre_groups, (N + kNetBlock - 1) / kNetBlock, size_t(resident_ ? res_.ctas : 0)});
  const size_t bm_words = pre_groups * (kNetBlock / 32);
  bitmask_.reset(3 * bm_words * 4);
  totals_.reset(groups * kTotalsStride * sizeof(unsigned long long));
  tick_dev_.reset(sizeof(long long));
  NGB_CUDA(cudaMemset(bitmask_.as<void>(), 0, 3 * bm_words * 4));
  NGB_CUDA(cudaMemset(totals_.as<void>(), 0, groups * kTotalsStride * sizeof(unsigned long long)));
  totals_pairs_ = groups;
  NGB_CUDA(cudaMemset(tick_dev_.as<void>(), 0, sizeof(long long)));
  d.bitmask = bitmask_.as<uint32_t>();
  d.bm_stride = int(bm_words);
  d.bm_bufs = 2;
  d.world = world_;
  d.rank = rank_;
  d.totals = totals_.as<unsigned long long>();
  // Split push shape: a CTA scans 64 bitmask words (2,048 presynaptic neurons)
  // when the presynaptic population is large, so the grid follows the spikes
  // rather than the population; lanes take 8 synapses a pass when this
  // partition's rows are short (under ~300 synapses on average), else 16.
  d.push_span_words = n_pre_ >= (1 << 20) ? 64 : 8;
  d.push_chunk = (n_pre_ > 0 && nnz_ / n_pre_ < 300) ? 8 : 16;
  // NEUROGEN_PUSH_SPAN = 8 | 64 and NEUROGEN_PUSH_CHUNK = 8 | 16 force the
  // shape (tests: results do not depend on it).
  if (const char *v = std::getenv("NEUROGEN_PUSH_SPAN")) d.push_span_words = std::atoi(v) == 64 ? 64 : 8;
  if (const char *v = std::getenv("NEUROGEN_PUSH_CHUNK")) d.push_chunk = std::atoi(v) == 8 ? 8 : 16;
  // Small networks: one fused launch per tick; large or partitioned: split
  // membrane / push, with the bitmask all-gather between them.
  split_ = world_ > 1 || c.launch == 2 || (c.launch == 0 && n_ >= 65536) || c.plasticity;
  if (c.plasticity) init_learning(bm_words);
  if (world_ > 1) {
    if (!nccl_id) throw std::invalid_argument("A partitioned network needs an NCCL unique id");
    ncclUniqueId id;
    std::memcpy(&id, nccl_id, sizeof id);
    nccl_check(nccl().CommInitRank(&comm_, world_, id, rank_), "ncclCommInitRank");
    NGB_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    if (world_ <= 32) setup_peer_exchange(bm_words); // one waiting lane per rank
  }
  if (!stream) NGB_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
  if (resident_) build_owner_blocks();
}

// One-sided spike exchange of a partitioned network (the default when every
// rank can map every other rank's memory; NEUROGEN_PEER_EXCHANGE=0 keeps the
// NCCL all-gather).  Each rank allocates its three bitmask buffers and its flag
// array in one block, shares the block's CUDA IPC handle with the others (one
// NCCL all-gather of fixed-size records that also carry the device's UUID and
// whether the rank wants the exchange), and maps theirs.  The decision is
// collective: one rank that cannot take part, or two ranks on the same GPU
// (whose waits could not run side by side), keeps every rank on NCCL.
void Network::setup_peer_exchange(size_t bm_words) {
  struct Record {
    int32_t ok;
    unsigned char uuid[16];
    cudaIpcMemHandle_t handle;
    int32_t pad[3];
  };
  const char *env = std::getenv("NEUROGEN_PEER_EXCHANGE");
  const size_t bm_bytes = 3 * bm_words * 4, flag_at = (bm_bytes + 255) & ~size_t(255);
  xbuf_.reset(flag_at + size_t(world_) * 8);
  NGB_CUDA(cudaMemset(xbuf_.as<void>(), 0, flag_at + size_t(world_) * 8));
  Record mine{};
  mine.ok = !(env && std::string(env) == "0");
  cudaDeviceProp prop{};
  NGB_CUDA(cudaGetDeviceProperties(&prop, device));
  std::memcpy(mine.uuid, &prop.uuid, 16);
  if (mine.ok && cudaIpcGetMemHandle(&mine.handle, xbuf_.as<void>()) != cudaSuccess) {
    (void)cudaGetLastError();
    mine.ok = 0;
  }
  auto gather = [&](const void *rec, size_t bytes, std::vector<unsigned char> &all) {
    DeviceBuffer buf(bytes * world_);
    NGB_CUDA(cudaMemcpy(buf.as<unsigned char>() + bytes * rank_, rec, bytes, cudaMemcpyHostToDevice));
    nccl_check(nccl().AllGather(buf.as<unsigned char>() + bytes * rank_, buf.as<void>(), bytes, ncclChar, comm_,
                                stream),
               "ncclAllGather (peer exchange set-up)");
    NGB_CUDA(cudaStreamSynchronize(stream));
    all.resize(bytes * world_);
    NGB_CUDA(cudaMemcpy(all.data(), buf.as<void>(), all.size(), cudaMemcpyDeviceToHost));
  };
  std::vector<unsigned char> all;
  gather(&mine, sizeof mine, all);
  std::vector<Record> recs(world_);
  std::memcpy(recs.data(), all.data(), all.size());
  bool ok = true;
  for (int r = 0; r < world_; ++r) {
    ok = ok && recs[r].ok;
    for (int q = 0; q < r; ++q) ok = ok && std::memcmp(recs[r].uuid, recs[q].uuid, 16) != 0;
  }
  std::vector<void *> base(world_, nullptr);
  base[rank_] = xbuf_.as<void>();
  int32_t opened = 1;
  if (ok) {
    for (int r = 0; r < world_ && opened; ++r) {
      if (r == rank_) continue;
      if (cudaIpcOpenMemHandle(&base[r], recs[r].handle, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        (void)cudaGetLastError();
        base[r] = nullptr;
        opened = 0;
      }
    }
  }
  // Second round: every rank mapped every other's block, or all fall back.
  std::vector<unsigned char> all_opened;
  gather(&opened, sizeof opened, all_opened);
  for (int r = 0; r < world_; ++r) ok = ok && reinterpret_cast<int32_t *>(all_opened.data())[r];
  if (!ok) {
    for (int r = 0; r < world_; ++r)
      if (r != rank_ && base[r]) cudaIpcCloseMemHandle(base[r]);
    xbuf_.reset(0);
    return;
  }
  peer_bases_ = base;
  std::vector<uint32_t *> bm(world_);
  std::vector<unsigned long long *> fl(world_);
  for (int r = 0; r < world_; ++r) {
    bm[r] = static_cast<uint32_t *>(base[r]);
    fl[r] = reinterpret_cast<unsigned long long *>(static_cast<unsigned char *>(base[r]) + flag_at);
  }
  peer_bm_ = upload_vec(bm);
  peer_flag_ = upload_vec(fl);
  xctl_.reset(16); // [0] error word, [2..3] epoch (u64)
  NGB_CUDA(cudaMemset(xctl_.as<void>(), 0, 16));
  NetDev &d = dev_;
  d.bitmask = bm[rank_];
  d.bm_bufs = 3;
  d.peer_bm = peer_bm_.as<uint32_t *>();
  d.peer_flag = peer_flag_.as<unsigned long long *>();
  d.xflag = fl[rank_];
  d.xerr = xctl_.as<int>();
  d.xepoch = reinterpret_cast<const unsigned long long *>(xctl_.as<unsigned>() + 2);
}

// A state load on a peer-exchange network is collective: every rank's earlier
// ticks are done (their kernels precede this all-gather on their streams), and
// the epoch advances, so flags stamped before the load never satisfy a wait
// after it, whatever tick the load sets.
void Network::exchange_epoch() {
  DeviceBuffer tmp(size_t(world_) * 4);
  nccl_check(nccl().AllGather(tmp.as<unsigned char>() + 4 * rank_, tmp.as<void>(), 4, ncclChar, comm_, stream),
             "ncclAllGather (state load)");
  NGB_CUDA(cudaStreamSynchronize(stream));
  ++epoch_;
  NGB_CUDA(cudaMemcpy(const_cast<unsigned long long *>(dev_.xepoch), &epoch_, 8, cudaMemcpyHostToDevice));
}

// Raises the peer exchange's error (a wait for another rank's spikes that ran out).
void Network::check_exchange() {
  if (!dev_.xerr) return;
  int err = 0;
  NGB_CUDA(cudaMemcpy(&err, dev_.xerr, 4, cudaMemcpyDeviceToHost));
  if (err) throw std::runtime_error("Peer spike exchange: a wait for another rank's spikes timed out");
}

// Learning buffers (biology.py:182-218): per CSR entry (padding included, never
// read) the pre trace (a stored contact's potential trace is the same value),
// coactivity and usage; per neuron the post trace, the rate and the scaling
// factor; the spike history; all zero.  Constants of the fp32 contract
// (oracle/net_oracle.c lc_of).
void Network::init_learning(size_t bm_words) {
  const ng_net_config &c = cfg;
  if (!dev_.row || dev_.bsr || (dev_.w_half && nnz_ > 0))
    throw std::invalid_argument("Learning needs fp32 weights in CSR storage");
  long long entries = 0;
  NGB_CUDA(cudaMemcpy(&entries, dev_.row + n_pre_, 8, cudaMemcpyDeviceToHost));
  const size_t E = size_t(std::max<long long>(entries, 1)), N = size_t(n_);
  for (DeviceBuffer *b : {&pre_tr_, &coact_, &usage_}) {
    b->reset(E * 4);
    NGB_CUDA(cudaMemset(b->as<void>(), 0, E * 4));
  }
  for (DeviceBuffer *b : {&post_tr_, &rate_, &scale_}) {
    b->reset(N * 4);
    NGB_CUDA(cudaMemset(b->as<void>(), 0, N * 4));
  }
  hist_.reset(size_t(kRingSlots) * bm_words * 4);
  NGB_CUDA(cudaMemset(hist_.as<void>(), 0, size_t(kRingSlots) * bm_words * 4));
  NetDev &d = dev_;
  d.pre_tr = pre_tr_.as<float>();
  d.coact = coact_.as<float>();
  d.usage = usage_.as<float>();
  d.post_tr = post_tr_.as<float>();
  d.rate = rate_.as<float>();
  d.scale = scale_.as<float>();
  d.hist = hist_.as<uint32_t>();
  d.learn_weights = 1;
  const double dt = c.dt_ms;
  d.l_decay = float(std::exp(-dt / 20.0));
  d.l_slow = float(std::exp(-dt / 1000.0));
  d.l_oms = float(1.0 - std::exp(-dt / 1000.0));
  d.l_rate_inc = float((1.0 - std::exp(-dt / 1000.0)) * 1000.0 / dt);
  d.l_per_ms = float(1000.0 / dt);
  d.l_alpha = float(2.0 * double(c.target_hz) * .020);
  d.l_stdp = c.stdp_rate;
  d.l_inh = c.inhibitory_rate;
  d.l_target = c.target_hz;
  d.l_tau_s = c.scaling_tau_ms;
  d.l_dt = float(dt);
}

// Learning state in the order of export_edges (CSR order, padding skipped).
void Network::plasticity_state(float *pre_tr, float *pot_tr, float *coact, float *usage, float *post_tr,
                               float *rate) {
  NGB_CUDA(cudaSetDevice(device));
  NGB_CUDA(cudaStreamSynchronize(stream));
  if (!dev_.pre_tr) throw std::invalid_argument("The network does not learn (plasticity = 0)");
  std::vector<long long> row(size_t(n_pre_) + 1);
  NGB_CUDA(cudaMemcpy(row.data(), row_.as<void>(), row.size() * 8, cudaMemcpyDeviceToHost));
  const size_t E = size_t(row[n_pre_]);
  std::vector<float> w(E), buf(E);
  if (E) NGB_CUDA(cudaMemcpy(w.data(), w_.as<void>(), E * 4, cudaMemcpyDeviceToHost));
  // The potential trace of a stored contact is its pre trace.
  const float *src[4] = {dev_.pre_tr, dev_.pre_tr, dev_.coact, dev_.usage};
  float *dst[4] = {pre_tr, pot_tr, coact, usage};
  for (int k = 0; k < 4; ++k) {
    if (!dst[k] || !E) continue;
    NGB_CUDA(cudaMemcpy(buf.data(), src[k], E * 4, cudaMemcpyDeviceToHost));
    size_t j = 0;
    for (size_t e = 0; e < E; ++e)
      if (w[e] != 0.f) dst[k][j++] = buf[e];
  }
  if (post_tr) NGB_CUDA(cudaMemcpy(post_tr, dev_.post_tr, size_t(n_) * 4, cudaMemcpyDeviceToHost));
  if (rate) NGB_CUDA(cudaMemcpy(rate, dev_.rate, size_t(n_) * 4, cudaMemcpyDeviceToHost));
}

// Resident launch plan: CTAs of P neurons (a multiple of 32, at least 256 so
// that small networks use few CTAs), one CTA per SM at most, shared memory for
// the state, a ring of Dr slots and the warps' event staging.  Returns false
// (or throws, when the resident launch was asked for) if it does not fit.
bool Network::plan_resident(int max_delay, bool required) {
  auto fail = [&](const std::string &why) -> bool {
    if (required) throw std::invalid_argument("Resident launch unavailable: " + why);
    return false;
  };
  int coop = 0, sms = 0, optin = 0;
  NGB_CUDA(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device));
  NGB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  NGB_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
  if (!coop) return fail("the device has no cooperative launch");
  int dr = 1;
  while (dr < max_delay) dr <<= 1;
  const bool ev64 = !dev_.bsr && dev_.w_half == 0; // fp16 weights (block storage is always fp16): 32-bit events
  int P = ((n_ + sms - 1) / sms + 31) / 32 * 32;
  P = std::max(P, std::min(256, (n_ + 31) / 32 * 32));
  if (const char *env = std::getenv("NEUROGEN_RESIDENT_PER_CTA")) P = std::max(P, (std::atoi(env) + 31) / 32 * 32);
  if (P > 2048) return fail("more than 2048 neurons per CTA (" + std::to_string(n_) + " neurons, " +
                            std::to_string(sms) + " SMs)");
  ResidentDev r{};
  r.per_cta = P;
  r.ctas = (n_ + P - 1) / P;
  r.ring_depth = dr;
  r.ev64 = ev64 ? 1 : 0;
  // Tick of the resident launch: NEUROGEN_RESIDENT_MODE=pipe | serial (the
  // default below), NEUROGEN_RESIDENT_MEMBER_WARPS=8 | 16 the pipelined tick's
  // membrane group.  The pipelined push addresses a CTA's rows by 32-bit
  // offsets from its first row.
  r.pipe = kResidentPipeDefault;
  if (const char *env = std::getenv("NEUROGEN_RESIDENT_MODE")) r.pipe = std::string(env) == "pipe" ? 1 : 0;
  if (!dev_.bsr && nnz_ + int64_t(kRowPad) * n_pre_ >= (int64_t(1) << 32)) r.pipe = 0;
  r.member_warps = 16;
  if (const char *env = std::getenv("NEUROGEN_RESIDENT_MEMBER_WARPS")) r.member_warps = std::atoi(env) == 8 ? 8 : 16;
  // Failure-path tests: an unreachable first barrier, so every CTA's bounded
  // wait runs out and the launch reports the error instead of running.
  if (const char *env = std::getenv("NEUROGEN_TEST_RESIDENT_STALL")) r.stall_test = std::atoi(env) ? 1 : 0;
  if (!ev64 && 2 * (dr + 1) * P >= 65536) return fail("ring offsets of " + std::to_string(P) + " neurons do not fit 16 bits");
  const size_t smem = resident_smem_bytes(r);
  if (smem + 2048 > size_t(optin)) // static shared memory and slack
    return fail(std::to_string(P) + " neurons a CTA with a " + std::to_string(dr) +
                "-slot ring need more shared memory than a CTA has");
  if (resident_max_ctas(r, dev_.bsr != 0, smem) < r.ctas)
    return fail("the device cannot hold " + std::to_string(r.ctas) + " resident CTAs at once");
  res_ = r;
  return true;
}

// Owner blocks from the device CSR or block storage: count the overflow
// blocks, allocate exactly, fill.
void Network::build_owner_blocks() {
  ResidentDev &r = res_;
  const size_t C = size_t(r.ctas);
  res_lists_.reset(3 * size_t(n_pre_) * 4);
  res_sync_.reset(16);
  res_err_.reset(4);
  NGB_CUDA(cudaMemset(res_sync_.as<void>(), 0, 16));
  NGB_CUDA(cudaMemset(res_err_.as<void>(), 0, 4));
  r.lists = res_lists_.as<int>();
  r.sync = res_sync_.as<unsigned>();
  r.err = res_err_.as<int>();
  DeviceBuffer scratch(16);
  unsigned long long *need = scratch.as<unsigned long long>(), *cursor = need + 1;
  NGB_CUDA(cudaMemsetAsync(need, 0, 16, stream));
  launch_owner_count(dev_, r, need, stream);
  NGB_CUDA(cudaGetLastError());
  unsigned long long overflow = 0;
  NGB_CUDA(cudaMemcpyAsync(&overflow, need, 8, cudaMemcpyDeviceToHost, stream));
  NGB_CUDA(cudaStreamSynchronize(stream));
  const unsigned long long total = (unsigned long long)n_pre_ * C + overflow;
  if (!r.ev64 && total >= 0x7FFFFFFFull) throw std::invalid_argument("Too many owner blocks for 32-bit events");
  const size_t bytes = size_t(total) * kOwnerBlockSlots * (r.ev64 ? 8 : 4);
  res_blocks_.reset(bytes);
  NGB_CUDA(cudaMemsetAsync(res_blocks_.as<void>(), 0xFF, bytes, stream));
  launch_owner_fill(dev_, r, res_blocks_.as<void>(), cursor, overflow, r.err, stream);
  NGB_CUDA(cudaGetLastError());
  int err = 0;
  unsigned long long used = 0;
  NGB_CUDA(cudaMemcpyAsync(&err, r.err, 4, cudaMemcpyDeviceToHost, stream));
  NGB_CUDA(cudaMemcpyAsync(&used, cursor, 8, cudaMemcpyDeviceToHost, stream));
  NGB_CUDA(cudaStreamSynchronize(stream));
  if (err || used != overflow) throw std::logic_error("Owner-block construction overflowed its allocation");
  r.blocks = res_blocks_.as<void>();
}

// Raises the resident kernel's error (a grid barrier that timed out).
void Network::check_resident() {
  if (!resident_) return;
  int err = 0;
  NGB_CUDA(cudaMemcpy(&err, res_.err, 4, cudaMemcpyDeviceToHost));
  if (err)
    throw std::runtime_error("Resident tick kernel: a grid barrier wait timed out; the network state is undefined");
}

Network::~Network() {
  if (graph_) cudaGraphExecDestroy(graph_); // before the communicator its NCCL nodes use
  for (size_t r = 0; r < peer_bases_.size(); ++r)
    if (int(r) != rank_ && peer_bases_[r]) cudaIpcCloseMemHandle(peer_bases_[r]);
  if (comm_) nccl().CommDestroy(comm_);
  for (cudaEvent_t e : {ev_fork_, ev_alif_, ev_rest_[0], ev_rest_[1], ev_join_})
    if (e) cudaEventDestroy(e);
  if (stream_rest_) cudaStreamDestroy(stream_rest_);
  if (stream) cudaStreamDestroy(stream);
}

// Membrane update of tick t (parity = t & 1, known on the host) and, for a
// partitioned network, the all-gather of the held slice of that tick's
// bitmask buffer into every rank's copy of the whole bitmask.
void Network::launch_membrane(TickRef t, int parity, uint32_t *spikes_row, unsigned long long *counts_row,
                              cudaStream_t st) {
  launch_net_alif(dev_, t, world_ > 1 ? nullptr : spikes_row, counts_row, st);
  if (world_ > 1) {
    uint32_t *bm;
    if (dev_.peer_bm) {
      // One-sided: the ranks' kernels have stored their slices here; wait for their flags.
      launch_net_xwait(dev_, t, st);
      bm = dev_.bitmask + size_t(t.t_dev ? 0 : t.k % 3) * size_t(dev_.bm_stride);
    } else {
      bm = bitmask_.as<uint32_t>() + size_t(parity) * size_t(dev_.bm_stride);
      const size_t words = size_t(n_) / 32;
      nccl_check(nccl().AllGather(bm + size_t(base_) / 32, bm, words, ncclUint32, comm_, st), "ncclAllGather");
    }
    if (spikes_row) // recorded runs only: the tick number is known here
      NGB_CUDA(cudaMemcpyAsync(spikes_row, bm, size_t(n_pre_) / 32 * 4, cudaMemcpyDeviceToDevice, st));
  }
}

// One whole tick in order on one stream (recorded runs, the ticks outside
// whole graph replays).
void Network::launch_tick(TickRef t, int parity, uint32_t *spikes_row, unsigned long long *counts_row,
                          cudaStream_t st) {
  if (split_) {
    launch_membrane(t, parity, spikes_row, counts_row, st);
    if (dev_.pre_tr) launch_net_learn(dev_, t, st); // learn before the tick's emissions (post traces: the push)
    launch_net_push(dev_, t, counts_row, 0, st);
  } else {
    launch_net_fused(dev_, t, spikes_row, counts_row, st);
  }
}

// One CUDA graph of kGraphTicks ticks reading the tick number from a device
// counter (advanced by the graph's last node); replays start on even ticks.
// Split networks run pipelined over two streams.  The membrane update and
// the delay-1 push of tick t stay on the main stream, since tick t+1 reads
// what they write.  The delay>=2 push of tick t runs on a second stream
// beside tick t+1: it writes ring slots t+2.. only, and its own counter
// slot.  Tick t+2's membrane update waits for it, because that tick reads
// ring slot t+2 and rewrites tick t's bitmask buffer.
void Network::capture_graph() {
  const long long *td = tick_dev_.as<long long>();
  const bool pipelined = split_ && !dev_.pre_tr; // learning: each tick's push before the next learns
  if (pipelined && !stream_rest_) {
    NGB_CUDA(cudaStreamCreateWithFlags(&stream_rest_, cudaStreamNonBlocking));
    for (cudaEvent_t *e : {&ev_fork_, &ev_alif_, &ev_rest_[0], &ev_rest_[1], &ev_join_})
      NGB_CUDA(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
  }
  cudaGraph_t g = nullptr;
  NGB_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
  try {
    if (pipelined) {
      NGB_CUDA(cudaEventRecord(ev_fork_, stream));
      NGB_CUDA(cudaStreamWaitEvent(stream_rest_, ev_fork_, 0));
      for (int k = 0; k < kGraphTicks; ++k) {
        const TickRef t{td, k};
        if (k >= 2) NGB_CUDA(cudaStreamWaitEvent(stream, ev_rest_[k & 1], 0));
        launch_membrane(t, k & 1, nullptr, nullptr, stream);
        NGB_CUDA(cudaEventRecord(ev_alif_, stream));
        launch_net_push(dev_, t, nullptr, 1, stream);
        NGB_CUDA(cudaStreamWaitEvent(stream_rest_, ev_alif_, 0));
        launch_net_push(dev_, t, nullptr, 2, stream_rest_);
        NGB_CUDA(cudaEventRecord(ev_rest_[k & 1], stream_rest_));
      }
      NGB_CUDA(cudaEventRecord(ev_join_, stream_rest_));
      NGB_CUDA(cudaStreamWaitEvent(stream, ev_join_, 0));
    } else {
      for (int k = 0; k < kGraphTicks; ++k) launch_tick(TickRef{td, k}, k & 1, nullptr, nullptr, stream);
    }
    launch_add_tick(tick_dev_.as<long long>(), kGraphTicks, stream);
  } catch (...) {
    cudaStreamEndCapture(stream, &g);
    if (g) cudaGraphDestroy(g);
    throw;
  }
  const cudaError_t e = cudaStreamEndCapture(stream, &g);
  if (e != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    cuda_check(e, "cudaStreamEndCapture");
  }
  const cudaError_t ie = cudaGraphInstantiate(&graph_, g, 0);
  cudaGraphDestroy(g);
  cuda_check(ie, "cudaGraphInstantiate");
}

void Network::stats(int64_t *totals) {
  NGB_CUDA(cudaSetDevice(device));
  NGB_CUDA(cudaDeviceSynchronize());
  check_resident();
  check_exchange();
  const size_t groups = totals_pairs_;
  std::vector<unsigned long long> g(groups * kTotalsStride);
  NGB_CUDA(cudaMemcpy(g.data(), totals_.as<void>(), g.size() * 8, cudaMemcpyDeviceToHost));
  totals[0] = totals[1] = 0;
  for (size_t k = 0; k < groups; ++k) {
    totals[0] += int64_t(g[kTotalsStride * k]);
    totals[1] += int64_t(g[kTotalsStride * k + 1]) + int64_t(g[kTotalsStride * k + 2]);
  }
}

void Network::export_edges(int32_t *pre, int32_t *post, int32_t *delay, float *weight) {
  NGB_CUDA(cudaSetDevice(device));
  Topology t;
  t.cfg = cfg;
  t.blocks = dev_.bsr != 0;
  if (t.blocks) {
    HostBSR &b = t.bsr;
    b.nb = n_ / 16;
    b.bcol.resize(size_t(b.nb) + 1);
    NGB_CUDA(cudaMemcpy(b.bcol.data(), bcol_.as<void>(), b.bcol.size() * 8, cudaMemcpyDeviceToHost));
    b.blk.resize(size_t(b.bcol[b.nb]));
    b.tiles.resize(b.blk.size() * 256);
    if (!b.blk.empty()) {
      NGB_CUDA(cudaMemcpy(b.blk.data(), blk_.as<void>(), b.blk.size() * 4, cudaMemcpyDeviceToHost));
      NGB_CUDA(cudaMemcpy(b.tiles.data(), tiles_.as<void>(), b.tiles.size() * 2, cudaMemcpyDeviceToHost));
    }
  } else {
    HostCSR &h = t.csr;
    h.n = n_pre_;
    h.post_base = base_;
    h.n_post = n_;
    h.row.resize(size_t(n_pre_) + 1);
    NGB_CUDA(cudaMemcpy(h.row.data(), row_.as<void>(), h.row.size() * 8, cudaMemcpyDeviceToHost));
    const size_t total = size_t(h.row[n_pre_]);
    h.syn.resize(total);
    if (total) NGB_CUDA(cudaMemcpy(h.syn.data(), syn_.as<void>(), total * 4, cudaMemcpyDeviceToHost));
    if (dev_.w_half) {
      h.w16.resize(total);
      if (total) NGB_CUDA(cudaMemcpy(h.w16.data(), w_.as<void>(), total * 2, cudaMemcpyDeviceToHost));
    } else {
      h.w32.resize(total);
      if (total) NGB_CUDA(cudaMemcpy(h.w32.data(), w_.as<void>(), total * 4, cudaMemcpyDeviceToHost));
    }
  }
  t.export_edges(pre, post, delay, weight);
}

void Network::set_state(const float *v, const float *a, const float *ge, const float *gi, const int32_t *ref,
                        const int32_t *ring, int64_t tick) {
  NGB_CUDA(cudaSetDevice(device));
  NGB_CUDA(cudaStreamSynchronize(stream));
  const size_t N = size_t(n_);
  if (v) NGB_CUDA(cudaMemcpy(v_.as<void>(), v, N * 4, cudaMemcpyHostToDevice));
  if (a) NGB_CUDA(cudaMemcpy(a_.as<void>(), a, N * 4, cudaMemcpyHostToDevice));
  if (ge) NGB_CUDA(cudaMemcpy(ge_.as<void>(), ge, N * 4, cudaMemcpyHostToDevice));
  if (gi) NGB_CUDA(cudaMemcpy(gi_.as<void>(), gi, N * 4, cudaMemcpyHostToDevice));
  if (ref) NGB_CUDA(cudaMemcpy(ref_.as<void>(), ref, N * 4, cudaMemcpyHostToDevice));
  if (ring) NGB_CUDA(cudaMemcpy(ring_.as<void>(), ring, size_t(kRingSlots) * N * 8, cudaMemcpyHostToDevice));
  if (tick < 0) throw std::invalid_argument("tick must be non-negative");
  tick_ = tick;
  if (dev_.peer_bm) exchange_epoch();
}

void Network::get_state(float *v, float *a, float *ge, float *gi, int32_t *ref, int32_t *ring, int64_t *tick) {
  NGB_CUDA(cudaSetDevice(device));
  NGB_CUDA(cudaStreamSynchronize(stream));
  check_resident();
  check_exchange();
  const size_t N = size_t(n_);
  if (v) NGB_CUDA(cudaMemcpy(v, v_.as<void>(), N * 4, cudaMemcpyDeviceToHost));
  if (a) NGB_CUDA(cudaMemcpy(a, a_.as<void>(), N * 4, cudaMemcpyDeviceToHost));
  if (ge) NGB_CUDA(cudaMemcpy(ge, ge_.as<void>(), N * 4, cudaMemcpyDeviceToHost));
  if (gi) NGB_CUDA(cudaMemcpy(gi, gi_.as<void>(), N * 4, cudaMemcpyDeviceToHost));
  if (ref) NGB_CUDA(cudaMemcpy(ref, ref_.as<void>(), N * 4, cudaMemcpyDeviceToHost));
  if (ring) NGB_CUDA(cudaMemcpy(ring, ring_.as<void>(), size_t(kRingSlots) * N * 8, cudaMemcpyDeviceToHost));
  if (tick) *tick = tick_;
}

void Network::enqueue(int ticks, uint32_t *d_spikes, unsigned long long *d_counts, cudaStream_t st) {
  if (ticks < 0) throw std::invalid_argument("ticks must be non-negative");
  const size_t words = (size_t(n_pre_) + 31) / 32;
  if (d_counts) NGB_CUDA(cudaMemsetAsync(d_counts, 0, size_t(ticks) * 16, st));
  if (resident_) {
    for (int k = 0; k < ticks;) {
      const int chunk = std::min(ticks - k, kResidentChunk);
      NGB_CUDA(cudaMemsetAsync(res_sync_.as<void>(), 0, 16, st));
      cuda_check(launch_net_resident(dev_, res_, tick_ + k, chunk, d_spikes ? d_spikes + size_t(k) * words : nullptr,
                                     d_counts ? d_counts + 2 * size_t(k) : nullptr, int(words), st),
                 "resident tick launch");
      k += chunk;
    }
    tick_ += ticks;
    return;
  }
  int k = 0;
  auto direct = [&](int kk) {
    const long long t = tick_ + kk;
    launch_tick(TickRef{nullptr, t}, int(t & 1), d_spikes ? d_spikes + size_t(kk) * words : nullptr,
                d_counts ? d_counts + 2 * size_t(kk) : nullptr, st);
  };
  const int lead = int(tick_ & 1); // graph replays start on even ticks
  if (!d_spikes && !d_counts && ticks - lead >= kGraphTicks) {
    if (lead) direct(k++);
    if (!graph_) capture_graph();
    launch_set_tick(tick_dev_.as<long long>(), tick_ + k, st);
    for (; k + kGraphTicks <= ticks; k += kGraphTicks) NGB_CUDA(cudaGraphLaunch(graph_, st));
  }
  for (; k < ticks; ++k) direct(k);
  NGB_CUDA(cudaGetLastError());
  tick_ += ticks;
}

void Network::run_host(int ticks, uint32_t *spikes, int64_t *counts) {
  NGB_CUDA(cudaSetDevice(device));
  const size_t words = (size_t(n_pre_) + 31) / 32;
  const int chunk = 1024;
  if (spikes) rec_spikes_.reset(size_t(std::min(ticks, chunk)) * words * 4 + 4);
  if (counts) rec_counts_.reset(size_t(std::min(ticks, chunk)) * 16 + 16);
  for (int done = 0; done < ticks; done += chunk) {
    const int k = std::min(chunk, ticks - done);
    enqueue(k, spikes ? rec_spikes_.as<uint32_t>() : nullptr,
            counts ? rec_counts_.as<unsigned long long>() : nullptr, stream);
    if (spikes)
      NGB_CUDA(cudaMemcpyAsync(spikes + size_t(done) * words, rec_spikes_.as<void>(), size_t(k) * words * 4,
                               cudaMemcpyDeviceToHost, stream));
    if (counts)
      NGB_CUDA(cudaMemcpyAsync(counts + 2 * size_t(done), rec_counts_.as<void>(), size_t(k) * 16,
                               cudaMemcpyDeviceToHost, stream));
    NGB_CUDA(cudaStreamSynchronize(stream));
    check_resident();
    check_exchange();
  }
  NGB_CUDA(cudaStreamSynchronize(stream));
}

} // namespace ngb
