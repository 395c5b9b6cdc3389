// Seeded input generators of the runtime (product side; the oracle has its
// own independent implementations and the tests compare the two).
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "../../include/apk.h"

namespace {

// glibc rand() (TYPE_3, the default state size), restated from the
// published description of its additive lagged-Fibonacci algorithm:
//   r[0] = seed (0 -> 1);  r[i] = 16807 * r[i-1] mod (2^31 - 1), i = 1..30
//   (computed with Schrage's method); r[i] = r[i-31], i = 31..33;
//   r[i] = r[i-31] + r[i-3] (mod 2^32), i >= 34;
//   the k-th output is r[k + 344] >> 1 (the first 310 values are skipped).
// The reference draws its inputs from this stream: src/persistent.cu:132-135.
class GlibcRand {
 public:
  explicit GlibcRand(unsigned seed) {
    int32_t r[34];
    r[0] = (int32_t)(seed == 0 ? 1 : seed);
    for (int i = 1; i < 31; ++i) {
      const int32_t hi = r[i - 1] / 127773;
      const int32_t lo = r[i - 1] % 127773;
      int32_t word = 16807 * lo - 2836 * hi;
      if (word < 0) word += 2147483647;
      r[i] = word;
    }
    for (int i = 31; i < 34; ++i) r[i] = r[i - 31];
    for (int i = 0; i < 34; ++i) ring_[i] = (uint32_t)r[i];
    pos_ = 34;
    for (int i = 34; i < 344; ++i) next_raw();
  }
  int next() { return (int)(next_raw() >> 1); }

 private:
  uint32_t next_raw() {
    // ring_ holds r[pos-34 .. pos-1] at index (j mod 34)
    const uint32_t v = ring_[(pos_ - 31) % 34] + ring_[(pos_ - 3) % 34];
    ring_[pos_ % 34] = v;
    ++pos_;
    return v;
  }
  uint32_t ring_[34];
  uint64_t pos_;
};

inline uint64_t splitmix64_at(uint64_t x) {
  uint64_t z = x + 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

inline uint16_t bf16_rne(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return (uint16_t)((u >> 16) | 0x40);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

}  // namespace

extern "C" {

void apk_fill_uniform(unsigned seed, float* A, size_t nA, float* B, size_t nB) {
  GlibcRand g(seed);
  const double rmax = 2147483647.0;  // RAND_MAX
  for (size_t i = 0; i < nA; ++i) A[i] = (float)(g.next() / rmax * 2.0 - 1.0);
  for (size_t i = 0; i < nB; ++i) B[i] = (float)(g.next() / rmax * 2.0 - 1.0);
}

// Element pair p: w0 = splitmix64(seed*2^32 + 2p), w1 = splitmix64(seed*2^32
// + 2p + 1); u1 = ((w0>>11)+1)*2^-53, u2 = (w1>>11)*2^-53; Box-Muller
// z0 = sqrt(-2 ln u1) cos(2 pi u2), z1 = ... sin(...); each -> float -> bf16.
void apk_fill_normal_bf16(unsigned long long seed, uint16_t* out, size_t n) {
  const uint64_t base = (uint64_t)seed << 32;
  auto work = [&](size_t lo, size_t hi) {
    const double two_pi = 6.283185307179586476925286766559;
    for (size_t i = lo; i < hi; i += 2) {
      const uint64_t p = i >> 1;
      const uint64_t w0 = splitmix64_at(base + 2 * p);
      const uint64_t w1 = splitmix64_at(base + 2 * p + 1);
      const double u1 = (double)((w0 >> 11) + 1) * 0x1.0p-53;
      const double u2 = (double)(w1 >> 11) * 0x1.0p-53;
      const double r = std::sqrt(-2.0 * std::log(u1));
      const double z0 = r * std::cos(two_pi * u2);
      const double z1 = r * std::sin(two_pi * u2);
      out[i] = bf16_rne((float)z0);
      if (i + 1 < n) out[i + 1] = bf16_rne((float)z1);
    }
  };
  unsigned nt = std::thread::hardware_concurrency();
  if (nt == 0) nt = 1;
  if (n < (1u << 20)) nt = 1;
  if (nt > 64) nt = 64;
  const size_t chunk = ((n + nt - 1) / nt + 1) & ~size_t(1);
  std::vector<std::thread> th;
  for (unsigned t = 0; t < nt; ++t) {
    const size_t lo = t * chunk;
    if (lo >= n) break;
    const size_t hi = lo + chunk < n ? lo + chunk : n;
    th.emplace_back(work, lo, hi);
  }
  for (auto& x : th) x.join();
}

void apk_round_bf16(const float* in, uint16_t* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = bf16_rne(in[i]);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// configs[4] task generator and static shard.

#include <algorithm>
#include <numeric>
#include <queue>
#include <random>

namespace {

// uniform double in [0,1) from one 64-bit draw
inline double u01(std::mt19937_64& g) { return (double)(g() >> 11) * 0x1.0p-53; }

int log_uniform_rounded(std::mt19937_64& g, int lo, int hi, int q) {
  const double x = std::exp(std::log((double)lo) + u01(g) * (std::log((double)hi) - std::log((double)lo)));
  int v = (int)std::floor(x / q + 0.5) * q;
  if (v < lo) v = lo;
  if (v > hi) v = hi;
  return v;
}

// uniform multiple of q in [0, hi] (hi >= 0)
int uniform_multiple(std::mt19937_64& g, int hi, int q) {
  const int slots = hi / q + 1;
  return (int)(g() % (unsigned long long)slots) * q;
}

}  // namespace

extern "C" {

long long apk_gen_tasks(unsigned long long seed, int n, int mn_lo, int mn_hi, int k_lo, int k_hi, int a_rows,
                        int a_cols, int b_rows, int b_cols, int c_rows, int c_cols, int n_samples,
                        apk_task* out) {
  std::mt19937_64 g(seed);
  const int sample_rows = 2048 * ((n_samples + 3) / 4);
  const int c_free_rows = c_rows - sample_rows;  // rows [0, c_free_rows) are shared by non-sampled tasks
  long long chk = 0;
  for (int t = 0; t < n; ++t) {
    apk_task& d = out[t];
    d.m = log_uniform_rounded(g, mn_lo, mn_hi, 128);
    d.n = log_uniform_rounded(g, mn_lo, mn_hi, 128);
    d.k = log_uniform_rounded(g, k_lo, k_hi, 64);
    const int tiles_m = (d.m + 255) / 256, tiles_n = d.n / 128;
    d.a_row0 = (int)(g() % (unsigned long long)(a_rows - tiles_m * 256 + 1));
    d.a_k0 = uniform_multiple(g, a_cols - d.k, 64);
    d.b_k0 = uniform_multiple(g, b_rows - d.k, 64);
    d.b_col0 = uniform_multiple(g, b_cols - d.n, 64);
    if (t < n_samples) {
      // disjoint 2048 x 2048 output windows that no other task touches
      d.c_row0 = c_free_rows + (t / 4) * 2048;
      d.c_col0 = (t % 4) * 2048;
      d.flags = APK_TASK_SAMPLED;
    } else {
      d.c_row0 = (int)(g() % (unsigned long long)(c_free_rows - d.m + 1));
      d.c_col0 = uniform_multiple(g, c_cols - d.n, 64);
      d.flags = 0;
    }
    d.chk_base = chk;
    chk += (long long)tiles_m * tiles_n;
  }
  return chk;
}

int apk_shard_tasks(const apk_task* tasks, int n, int world, int rank, int* idx) {
  if (world <= 1) {
    for (int t = 0; t < n; ++t) idx[t] = t;
    return n;
  }
  std::vector<int> order(n);
  std::iota(order.begin(), order.end(), 0);
  auto flops = [&](int t) { return 2.0 * tasks[t].m * tasks[t].n * (double)tasks[t].k; };
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return flops(a) > flops(b); });
  // least-loaded rank first; ties to the lowest rank
  using Load = std::pair<double, int>;
  std::priority_queue<Load, std::vector<Load>, std::greater<Load>> heap;
  for (int r = 0; r < world; ++r) heap.push({0.0, r});
  std::vector<int> owner(n);
  for (int t : order) {
    Load l = heap.top();
    heap.pop();
    owner[t] = l.second;
    l.first += flops(t);
    heap.push(l);
  }
  int m = 0;
  for (int t = 0; t < n; ++t)
    if (owner[t] == rank) idx[m++] = t;
  return m;
}

}  // extern "C"
