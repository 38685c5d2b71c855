// Host simulation of the tensor-parallel reduce-scatter / all-gather flag protocol.
//
// The device protocol (csrc/kernels/comm.cu rs_norm_ag_kernel, with the scatter epilogue of
// csrc/kernels/gemm_tcgen05.cu) runs here with ranks and CTAs as threads and the PTX operations as
// C++ atomics of the same strength:
//   producer CTA (GEMM epilogue)  plain stores of partial rows into the owner's receive buffer, then
//                                 fence.acq_rel.sys + red.relaxed.sys.add on the owner's rs counter
//                                 -> std::atomic fetch_add(release)
//   consumer CTA (rs_norm_ag)     ld.acquire.sys spin on the rs counter up to state[0] + rs_inc
//                                 -> load(acquire) in a bounded loop; sums its owned rows; pushes
//                                 them into every rank's h (plain stores); fence + red.add on every
//                                 rank's ag counter -> fetch_add(release); atom.acq_rel.gpu on the
//                                 site's CTA counter, the last CTA advancing the targets
//                                 (state[0], state[1]) of the next call; CTA 0 waits for its own ag
//                                 counter before the kernel ends.
//   kernel boundaries             a barrier among a rank's CTA threads (stream order).
// Counters only grow; targets advance by the arrivals of one call; the receive buffers and h are
// reused by every call, so a missing happens-before edge shows up as a wrong sum (the result is
// compared with a serial computation of the same layers) or, in the ThreadSanitizer build, as a
// reported race. Random delays between the steps shuffle the interleavings. Waits are bounded and
// report which wait gave up instead of hanging.
//
//   vmc_tp_protocol_sim RANKS CTAS LAYERS SEED [MUTATION]
//
// MUTATION weakens one step on purpose, to show that the simulation notices: "relaxed-signal" (the
// producers' arrival without release), "no-ag-wait" (the kernel ends without waiting for the
// all-gather), "early-advance" (the first CTA instead of the last advances the targets).
#include <atomic>
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <memory>
#include <random>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace {

constexpr int kH = 16;        // hidden size (elements per row)
constexpr int kRowsPerRank = 6;
constexpr int kSites = 2;     // two row-parallel sites per layer (attention output, FFN down)
constexpr int kSplits = 2;    // K splits: each source rank sends two partial tiles per owner row

// A reusable barrier for one rank's CTA threads (the end of a kernel on that rank's stream). It
// gives up once the run has failed, so that a failed wait ends the run instead of hanging it.
class Barrier {
 public:
  Barrier(int n, const std::atomic<int>& failed) : n_(n), failed_(failed) {}
  void wait() {
    const int gen = gen_.load(std::memory_order_acquire);
    if (count_.fetch_add(1, std::memory_order_acq_rel) + 1 == n_) {
      count_.store(0, std::memory_order_relaxed);
      gen_.fetch_add(1, std::memory_order_acq_rel);
    } else {
      while (gen_.load(std::memory_order_acquire) == gen && !failed_.load(std::memory_order_relaxed))
        std::this_thread::yield();
    }
  }

 private:
  const int n_;
  const std::atomic<int>& failed_;
  std::atomic<int> count_{0}, gen_{0};
};

struct RankMem {
  // receive buffers of the two sites: [slot = source rank * kSplits + split][owned row][kH]
  std::vector<uint32_t> recv[kSites];
  std::vector<uint32_t> h, resid;  // [T][kH]: h is all-gathered, resid rows owned by this rank
  std::atomic<uint32_t> rs_count[kSites];
  std::atomic<uint32_t> ag_count[kSites];
  uint32_t state[kSites][2] = {};      // rs target, ag target (this rank's private bookkeeping)
  std::atomic<uint32_t> done[kSites];  // CTAs of the current call that finished (state[2])
};

struct Sim {
  int NR, G, L, T;
  uint32_t seed;
  std::string mutation;
  std::vector<std::unique_ptr<RankMem>> r;
  std::atomic<int> failed{0};
  std::atomic<uint64_t> max_wait_polls{0};

  // deterministic "GEMM" and "norm" of the simulation: integer functions so sums are exact
  static uint32_t partial(uint32_t hv, int layer, int site, int src, int split, int row, int e) {
    uint32_t x = hv * 2654435761u + static_cast<uint32_t>(layer * 97 + site * 31 + src * 7 + split * 3 + row * 5 + e);
    x ^= x >> 13;
    return x * 0x9E3779B1u;
  }
  static uint32_t norm(uint32_t s, int layer, int site) { return (s ^ (s >> 7)) + static_cast<uint32_t>(layer + site); }

  void delay(std::mt19937& rng) {
    const uint32_t d = rng() % 16;
    if (d < 10) return;
    if (d < 14) std::this_thread::yield();
    else std::this_thread::sleep_for(std::chrono::microseconds(rng() % 50));
  }

  bool wait_at_least(const std::atomic<uint32_t>& c, uint32_t target, const char* what, int rank) {
    const auto t0 = std::chrono::steady_clock::now();
    for (uint64_t i = 0;; ++i) {
      if (static_cast<int32_t>(c.load(std::memory_order_acquire) - target) >= 0) {
        uint64_t m = max_wait_polls.load(std::memory_order_relaxed);
        while (i > m && !max_wait_polls.compare_exchange_weak(m, i)) {
        }
        return true;
      }
      if (failed.load(std::memory_order_relaxed)) return false;
      if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(5)) {
        fprintf(stderr, "rank %d gave up waiting on %s (target %u, value %u)\n", rank, what, target,
                c.load(std::memory_order_relaxed));
        failed.store(1);
        return false;
      }
      if (i > 64) std::this_thread::yield();
    }
  }

  // One CTA thread `b` of rank `me`.
  void cta(int me, int b, Barrier& bar) {
    std::mt19937 rng(seed * 1000003u + static_cast<uint32_t>(me * 131 + b));
    RankMem& m = *r[me];
    const int rpr = kRowsPerRank;
    // producer CTAs: CTA b sends the tiles of the owners o with o % G == b (every row and K split of
    // each), then signals each of those owners once: NR arrivals per owner and call
    for (int layer = 0; layer < L && !failed.load(); ++layer) {
      for (int site = 0; site < kSites && !failed.load(); ++site) {
        // ---- GEMM with scatter epilogue (one kernel) ----
        for (int o = b; o < NR; o += G) {
          RankMem& own = *r[o];
          for (int split = 0; split < kSplits; ++split) {
            for (int lr = 0; lr < rpr; ++lr) {
              const int row = o * rpr + lr;
              uint32_t* dst = own.recv[site].data() + (static_cast<size_t>(me * kSplits + split) * rpr + lr) * kH;
              for (int e = 0; e < kH; ++e)
                dst[e] = partial(m.h[static_cast<size_t>(row) * kH + e], layer, site, me, split, row, e);
            }
            delay(rng);
          }
          own.rs_count[site].fetch_add(1, mutation == "relaxed-signal" ? std::memory_order_relaxed
                                                                        : std::memory_order_release);
        }
        bar.wait();  // kernel boundary
        // ---- rs_norm_ag (one kernel) ----
        const uint32_t arrivals = static_cast<uint32_t>(NR);  // one producer CTA per (source rank, owner)
        if (!wait_at_least(m.rs_count[site], m.state[site][0] + arrivals, "the reduce-scatter arrivals", me)) break;
        for (int lr = b; lr < rpr; lr += G) {
          const int row = me * rpr + lr;
          for (int e = 0; e < kH; ++e) {
            uint32_t s = m.resid[static_cast<size_t>(row) * kH + e];
            for (int sl = 0; sl < NR * kSplits; ++sl) s += m.recv[site][(static_cast<size_t>(sl) * rpr + lr) * kH + e];
            m.resid[static_cast<size_t>(row) * kH + e] = s;
            const uint32_t out = norm(s, layer, site);
            for (int q = 0; q < NR; ++q) {
              r[(me + q) % NR]->h[static_cast<size_t>(row) * kH + e] = out;  // push into every rank's h
            }
          }
          delay(rng);
        }
        const uint32_t ag_inc = static_cast<uint32_t>(NR * G);
        const uint32_t ag_target = m.state[site][1] + ag_inc;  // read before this CTA counts itself
        for (int q = 0; q < NR; ++q) r[q]->ag_count[site].fetch_add(1, std::memory_order_release);
        const uint32_t old = m.done[site].fetch_add(1, std::memory_order_acq_rel);
        if (old == (mutation == "early-advance" ? 0u : static_cast<uint32_t>(G - 1))) {  // the last CTA advances
          m.state[site][0] += arrivals;
          m.state[site][1] += ag_inc;
          m.done[site].store(0, std::memory_order_relaxed);
        }
        if (b == 0 && mutation != "no-ag-wait" &&
            !wait_at_least(m.ag_count[site], ag_target, "the all-gather arrivals", me))
          break;
        bar.wait();  // kernel boundary
      }
    }
  }

  // the same layers on one thread
  std::vector<uint32_t> serial() const {
    std::vector<uint32_t> h(static_cast<size_t>(T) * kH), resid(static_cast<size_t>(T) * kH);
    for (int i = 0; i < T * kH; ++i) {
      h[i] = static_cast<uint32_t>(i * 7 + 1);
      resid[i] = static_cast<uint32_t>(i * 3);
    }
    for (int layer = 0; layer < L; ++layer)
      for (int site = 0; site < kSites; ++site) {
        std::vector<uint32_t> nh(h.size());
        for (int row = 0; row < T; ++row)
          for (int e = 0; e < kH; ++e) {
            uint32_t s = resid[static_cast<size_t>(row) * kH + e];
            for (int src = 0; src < NR; ++src)
              for (int split = 0; split < kSplits; ++split)
                s += partial(h[static_cast<size_t>(row) * kH + e], layer, site, src, split, row, e);
            resid[static_cast<size_t>(row) * kH + e] = s;
            nh[static_cast<size_t>(row) * kH + e] = norm(s, layer, site);
          }
        h.swap(nh);
      }
    return h;
  }
};

}  // namespace

int main(int argc, char** argv) {
  if (argc != 5 && argc != 6) {
    fprintf(stderr, "usage: vmc_tp_protocol_sim RANKS CTAS LAYERS SEED [MUTATION]\n");
    return 2;
  }
  Sim s;
  s.NR = atoi(argv[1]);
  s.G = atoi(argv[2]);
  s.L = atoi(argv[3]);
  s.seed = static_cast<uint32_t>(atoi(argv[4]));
  s.mutation = argc == 6 ? argv[5] : "";
  if (s.NR < 1 || s.NR > 8 || s.G < 1 || s.G > 8 || s.L < 1) {
    fprintf(stderr, "bad arguments\n");
    return 2;
  }
  s.T = s.NR * kRowsPerRank;
  for (int q = 0; q < s.NR; ++q) {
    auto m = std::make_unique<RankMem>();
    for (int site = 0; site < kSites; ++site) {
      m->recv[site].assign(static_cast<size_t>(s.NR) * kSplits * kRowsPerRank * kH, 0u);
      m->rs_count[site].store(0);
      m->ag_count[site].store(0);
      m->done[site].store(0);
    }
    m->h.resize(static_cast<size_t>(s.T) * kH);
    m->resid.resize(static_cast<size_t>(s.T) * kH);
    for (int i = 0; i < s.T * kH; ++i) {
      m->h[i] = static_cast<uint32_t>(i * 7 + 1);
      m->resid[i] = static_cast<uint32_t>(i * 3);
    }
    s.r.push_back(std::move(m));
  }
  std::vector<std::unique_ptr<Barrier>> bars;
  for (int q = 0; q < s.NR; ++q) bars.push_back(std::make_unique<Barrier>(s.G, s.failed));
  std::vector<std::thread> th;
  for (int q = 0; q < s.NR; ++q)
    for (int b = 0; b < s.G; ++b) th.emplace_back([&s, &bars, q, b] { s.cta(q, b, *bars[q]); });
  for (auto& t : th) t.join();
  if (s.failed.load()) {
    printf("{\"ok\": false, \"reason\": \"a bounded wait gave up\"}\n");
    return 1;
  }
  const auto want = s.serial();
  int bad = 0;
  for (int q = 0; q < s.NR; ++q)
    for (size_t i = 0; i < want.size(); ++i) bad += s.r[q]->h[i] != want[i];
  printf("{\"ok\": %s, \"ranks\": %d, \"ctas\": %d, \"layers\": %d, \"mismatches\": %d, \"max_wait_polls\": %llu}\n",
         bad ? "false" : "true", s.NR, s.G, s.L, bad, static_cast<unsigned long long>(s.max_wait_polls.load()));
  return bad ? 1 : 0;
}
