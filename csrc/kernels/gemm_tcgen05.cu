// Fused-dequant GEMM on the 5th-generation tensor cores: out[M, N] = X[M, K] @ W[N, K]^T.
//
// B200-native replacement for the reference's quantized matmul path (ggml-cuda mul_mat_q /
// mul_mat_vec_q, ggml-cuda/mmq.cuh:3542, mmvq.cu:398, and cuBLAS for F16/BF16 weights), which on
// sm_100 runs as Ampere-class mma.sync / dp4a code.
//
// Design ("swap-AB", persistent, warp-specialised). The weight tile is the UMMA A operand
// (M_mma = 128 output features), the activation tile is the B operand (N_mma = BN tokens, 16..256),
// and the fp32 accumulator lives in TMEM, double-buffered so that the epilogue of one work unit
// overlaps the main loop of the next. A work unit is (128-feature tile, BN-token tile, K split);
// one CTA per SM walks the units round-robin, so the weight stream never drains between tiles.
// Warp roles in a 480-thread CTA:
//   warp 0      weight producer: one cp.async.bulk per weight tile (tiles are stored contiguously,
//               see weight_formats.cuh) into the raw ring, or straight into the A ring for bf16.
//               Weights do not depend on the previous kernel, so the first tiles are requested
//               before the programmatic-dependency wait.
//   warp 1      allocates TMEM; one elected lane issues tcgen05.mma (K=16 per instruction) and
//               tcgen05.commit to release ring stages and hand finished accumulators over.
//   warps 2-9   dequantize GGUF blocks from the raw ring into the 128B-swizzled bf16 A ring
//               (packed bf16x2 integer tricks, see the per-format functions).
//   warp 10     activation producer: TMA 2-D loads (128B swizzle, zero fill past M / K).
//   warps 11-14 epilogue: tcgen05.ld -> bf16 store, fp32 store (per-split partials, no atomics),
//               fp32 red.add, or the fused SwiGLU (gate / up rows interleaved).
// Every wait is bounded; on expiry the CTA records an error code and unwinds (TMEM is freed).
#include <cuda.h>

#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "gemm_tcgen05.h"
#include "weight_formats.cuh"

namespace vmc {
namespace {

constexpr int kThreads = 480;
constexpr int kDequantWarps = 8;
constexpr int kFirstDqWarp = 2;
constexpr int kBWarp = 10;
constexpr int kFirstEpiWarp = 11;

struct GemmSmemPlan {
  int a_stages = 0;    // A (weights, bf16 swizzled) ring stages, 64-K each
  int b_stages = 0;    // B (activations) ring stages, 64-K each
  int raw_stages = 0;  // raw quant tile stages (one chunk = 256-K each)
  int bn = 0;
  int wf = 0;
  __host__ __device__ constexpr int a_bytes() const { return 128 * 128; }
  __host__ __device__ constexpr int b_bytes() const { return bn * 128; }
  __host__ __device__ constexpr int raw_bytes() const { return wf == kWfBF16 ? 0 : wf_tile_bytes(wf); }
  __host__ __device__ constexpr int off_b() const { return a_stages * a_bytes(); }
  __host__ __device__ constexpr int off_raw() const { return off_b() + b_stages * b_bytes(); }
  __host__ __device__ constexpr int off_bar() const { return off_raw() + raw_stages * raw_bytes(); }
  __host__ __device__ constexpr int nbars() const { return 2 * a_stages + 2 * b_stages + 2 * raw_stages + 4; }
  __host__ __device__ constexpr int total() const { return off_bar() + nbars() * 8 + 16 + 1024; }
};

// Shared-memory plan for one CTA per SM. The A and B rings are independent so that each can be as
// deep as its producer's latency needs: the activation ring (TMA from L2) is made deep for
// decode-sized tiles, the raw weight ring (HBM) next, and the dequantised A ring stays short
// because its producer (the dequant warps) sits next to the consumer.
__host__ __device__ constexpr GemmSmemPlan make_plan(int wf, int bn) {
  GemmSmemPlan p;
  p.bn = bn;
  p.wf = wf;
  const int budget = 222 * 1024;
  const bool quant = wf != kWfBF16;
  p.b_stages = 2;
  p.raw_stages = quant ? 2 : 0;
  // Quantized formats: the dequant warps fill A one 64-K stage at a time, so any ring of at least
  // one chunk (4 stages) works.
  p.a_stages = quant ? 8 : 2;
  if (quant && p.total() > budget) {
    // Wide token tiles: one chunk of A stages (the dequant warps hand stages over one at a time)
    // and a third activation stage. Measured on the 8B prefill shapes with BN = 256: A 4 / B 3 /
    // raw 3 runs the down projection at 1068 TFLOP/s where A 6 / B 2 / raw 3 ran it at 748.
    p.a_stages = 4;
    p.b_stages = 3;
    if (p.total() > budget) p.b_stages = 2;  // formats with large raw tiles
  }
  const int b_cap = bn <= 64 ? 16 : 6;
  bool grew = true;
  while (grew) {
    grew = false;
    if (p.b_stages < b_cap) {
      GemmSmemPlan q = p;
      q.b_stages += 1;
      if (q.total() <= budget) { p = q; grew = true; }
    }
    if (quant && p.raw_stages < 6) {
      GemmSmemPlan q = p;
      q.raw_stages += 1;
      if (q.total() <= budget) { p = q; grew = true; }
    }
    if (!quant && p.a_stages < 8) {
      GemmSmemPlan q = p;
      q.a_stages += 1;
      if (q.total() <= budget) { p = q; grew = true; }
    }
  }
  return p;
}

// ---------------------------------------------------------------------------------------------
// Dequantizers: thread (row r, half h) of substep s (64 K-elements) produces 32 bf16 values =
// 16 packed words, elements [64s + 32h, 64s + 32h + 32) of the 256-wide chunk.

__device__ __forceinline__ uint32_t bf2_sub(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hsub2(*reinterpret_cast<__nv_bfloat162*>(&a), *reinterpret_cast<__nv_bfloat162*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t bf2_fma(uint32_t a, uint32_t b, uint32_t c) {
  __nv_bfloat162 r = __hfma2(*reinterpret_cast<__nv_bfloat162*>(&a), *reinterpret_cast<__nv_bfloat162*>(&b),
                             *reinterpret_cast<__nv_bfloat162*>(&c));
  return *reinterpret_cast<uint32_t*>(&r);
}
// Single-instruction forms for the dequant inner loops. Measured on B200: the bit operations and
// the packed bf16 ops each issue at 2 warp-instructions per cycle per SM, and the generic
// __nv_bfloat162 helpers above cost the integer pipe extra instructions on this toolchain.
__device__ __forceinline__ uint32_t lop_and_or(uint32_t x, uint32_t m, uint32_t c) {  // (x & m) | c
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(x), "r"(m), "r"(c));
  return r;
}
__device__ __forceinline__ uint32_t bsub2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t bmul2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t bfma2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

constexpr uint32_t kMagic128x2 = 0x43004300u;  // bf16 (128, 128); 128 + q is exact for q < 128

// Per-chunk Q4_K state of thread (row, half): bf16x2 scale and negated min of its four sub-blocks
// j = 2s + h (s = 0..3), decoded once per 256-K chunk instead of once per 64-K substep.
struct Q4KChunk {
  uint32_t ds2[4], ndm2[4];
};
__device__ __forceinline__ void q4k_prep(const uint8_t* row, int h, Q4KChunk& c) {
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(row + 4 * (2 * s + h));  // (ds, ndm) of sub-block j
    c.ds2[s] = __byte_perm(w, 0u, 0x1010);
    c.ndm2[s] = __byte_perm(w, 0u, 0x3232);
  }
}
__device__ __forceinline__ void q4k_sub(const uint8_t* row, int s, int h, const Q4KChunk& c, uint32_t (&o)[16]) {
  const uint4* q = reinterpret_cast<const uint4*>(row + 32 + 32 * s);
  const uint4 w0 = q[0], w1 = q[1];
  const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
  const uint32_t ds2 = c.ds2[s], ndm2 = c.ndm2[s];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t lo = h ? (w[i] >> 4) : w[i];
    const uint32_t p01 = (lo & 0x000f000fu) | kMagic128x2;
    const uint32_t p23 = ((lo >> 8) & 0x000f000fu) | kMagic128x2;
    o[2 * i] = bf2_fma(bf2_sub(p01, kMagic128x2), ds2, ndm2);
    o[2 * i + 1] = bf2_fma(bf2_sub(p23, kMagic128x2), ds2, ndm2);
  }
}

__device__ __forceinline__ void dq_q6k(const uint8_t* row, int s, int h, uint32_t (&o)[16]) {
  const int g8 = 8 * s + 4 * h;   // first 8-element group of this thread
  const int g16 = 4 * s + 2 * h;  // first 16-element group
  const uint4 lo = *reinterpret_cast<const uint4*>(row + 4 * g8);
  const uint2 hi = *reinterpret_cast<const uint2*>(row + 128 + 4 * g16);
  const uint32_t scw = *reinterpret_cast<const uint32_t*>(row + 192 + 2 * g16);
  const uint32_t sc0 = (scw & 0xffffu) * 0x10001u;  // bf16x2 splat of group scale
  const uint32_t sc1 = (scw >> 16) * 0x10001u;
  const uint32_t lw[4] = {lo.x, lo.y, lo.z, lo.w};
  const uint32_t kOff = 0x43204320u;  // bf16 (160, 160) = 128 + 32
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t V = (i < 2) ? hi.x : hi.y;
    const uint32_t scale = (i < 2) ? sc0 : sc1;
    const int kb = (i & 1) * 4;  // pair index base inside the 16-element group
    const uint32_t W = lw[i];
    const uint32_t nib[4] = {W & 0x000f000fu, (W >> 8) & 0x000f000fu, (W >> 4) & 0x000f000fu, (W >> 12) & 0x000f000fu};
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const int k = kb + p;
      const int sh = 2 * k - 4;
      const uint32_t hb = (sh >= 0 ? (V >> sh) : (V << (-sh))) & 0x00300030u;
      const uint32_t x = nib[p] | hb | kMagic128x2;
      o[4 * i + p] = bmul2(bsub2(x, kOff), scale);
    }
  }
}

__device__ __forceinline__ void dq_q8_0(const uint8_t* row, int s, int h, uint32_t (&o)[16]) {
  const int b = 2 * s + h;
  const uint32_t d = *reinterpret_cast<const uint16_t*>(row + 2 * b);
  const uint32_t d2 = d * 0x10001u;
  const uint4* q = reinterpret_cast<const uint4*>(row + 16 + 32 * b);
  const uint4 w0 = q[0], w1 = q[1];
  const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    // Bytes stored (q0,q2,q1,q3): each masked half holds one two's-complement byte B = 128*b7 + low7.
    // (128 + low7) is exact in bf16; q = B (b7 clear) or B - 256 (b7 set), so the subtrahend is
    // 128 (0x4300) or 256 (0x4380), selected by copying b7 into the mantissa's top bit.
    const uint32_t x01 = w[i], x23 = w[i] >> 8;
    const uint32_t y01 = (x01 & 0x007f007fu) | kMagic128x2;
    const uint32_t z01 = (x01 & 0x00800080u) | kMagic128x2;
    const uint32_t y23 = (x23 & 0x007f007fu) | kMagic128x2;
    const uint32_t z23 = (x23 & 0x00800080u) | kMagic128x2;
    o[2 * i] = bmul2(bsub2(y01, z01), d2);
    o[2 * i + 1] = bmul2(bsub2(y23, z23), d2);
  }
}

// ---------------------------------------------------------------------------------------------

struct GemmArgs {
  const uint8_t* w;       // tiled weights
  int N, K, M;
  int KC;                 // number of K chunks in the tiled weight (ceil(K / chunk))
  int chunks_per_split;
  int n_tiles, m_tiles, splits;
  int units;              // n_tiles * m_tiles * splits
  void* out;
  int ldo;                // output row stride in elements
  int64_t split_stride;   // elements between the per-split output slices (kGemmOutF32Split)
  int out_mode;           // GemmOut
  uint32_t* err;
  unsigned long long* trace;  // optional per-role timestamps of CTA 0 (diagnostics), else null
  int bn;                     // token tile width
  // Grouped mode (groups > 0, e.g. MoE experts): group g owns rows [offset[g], offset[g] + count[g])
  // of X and of the output (device arrays, read by the kernel) and the weight at w + g * w_stride.
  // m_tiles is then the per-group tile bound; units past a group's count are skipped by every role.
  int groups;
  const int32_t* grp_count;
  const int32_t* grp_offset;
  int64_t grp_w_stride;  // bytes
  // Scatter mode (kGemmOutScatterBF16: the reduce-scatter of a tensor-parallel row-parallel GEMM):
  // output row m belongs to rank o = m / scat_rpr and is stored (bf16) as row m - o * scat_rpr of
  // slot (scat_rank * splits + split) of that rank's receive buffer scat[o] (row stride ldo, slots
  // scat_rpr rows apart). When a CTA has stored all its units it releases them (barrier over the
  // epilogue warps, system-scope fence) and counts itself on scat_local, a counter in this GPU's
  // memory; the last of the grid's CTAs then adds 1 to every rank's arrival counter scat_count[o]
  // (one arrival per source rank and call: a peer's counter takes N remote atomics, not N x grid).
  // Without scat_local every CTA adds to every rank's counter.
  void* scat[8];
  uint32_t* scat_count[8];
  uint32_t* scat_local;
  int scat_rpr, scat_rank, scat_nranks;
  // Row-scatter mode (kGemmOutRowScatterBF16, the combine of an expert-parallel MoE layer): output
  // row m goes to the rank, row and top-k slot packed in row_ret[m] ((rank << 24) | (row << 3) | j):
  // row (row * row_k + j) of that rank's buffer scat[rank] (row stride ldo); release / arrival as in
  // scatter mode. Rows whose return word is negative are skipped.
  const int32_t* row_ret;
  int row_k;
  // Stream-K (decode kernel, one token tile, no K split): CTA b of G takes chunks
  // [b * W / G, (b + 1) * W / G) of the W = n_tiles * KC sequence (weight tile, 256-K chunk), cut
  // into segments at tile borders. A tile split across CTAs is finished by the CTA holding its chunk 0
  // (its last segment): the later CTAs store their fp32 partial accumulators into their slot of sk_ws
  // ([G][BN][128]) and count on sk_cnt[tile]; the finisher waits for the count, adds the partials in
  // CTA order and runs the normal epilogue, then resets the count.
  int sk;
  float* sk_ws;
  uint32_t* sk_cnt;
};

__device__ __forceinline__ void epi_bar_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Reduce-scatter epilogue of 16 consecutive rows m_base .. m_base + 15 (column n) of a unit.
__device__ __forceinline__ void scatter_rows(const GemmArgs& a, int split, int n, int m_base, int m_end,
                                             const uint32_t (&v)[16]) {
  const int rpr = a.scat_rpr;
  int o = m_base / rpr;
  int lr = m_base - o * rpr;
  const size_t slot = static_cast<size_t>(a.scat_rank * a.splits + split) * rpr;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    if (m_base + j < m_end) {
      __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(a.scat[o]) + (slot + lr) * a.ldo + n;
      *dst = __float2bfloat16(__uint_as_float(v[j]));
    }
    if (++lr == rpr) {
      lr = 0;
      ++o;
    }
  }
}

// Expert-parallel combine epilogue: each row goes back to the rank and slot its token came from.
__device__ __forceinline__ void row_scatter_rows(const GemmArgs& a, int n, int m_base, int m_end,
                                                 const uint32_t (&v)[16]) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int m = m_base + j;
    if (m < m_end) {
      const int32_t ret = a.row_ret[m];
      if (ret >= 0) {
        const int src = ret >> 24, row = (ret >> 3) & 0x1fffff, slot = ret & 7;
        __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(a.scat[src]) +
                             (static_cast<size_t>(row) * a.row_k + slot) * a.ldo + n;
        *dst = __float2bfloat16(__uint_as_float(v[j]));
      }
    }
  }
}

// After a CTA's last unit: make its peer stores visible (system-scope fence), then count the arrival.
// Hierarchical (scat_local set): each CTA adds itself to the local counter with a GPU-scope acq_rel
// atomic; the CTA that completes the grid resets it, and its system-scope fence orders every CTA's
// stores (acquired through the local counter) before its one arrival at each rank.
__device__ __forceinline__ void scatter_release(const GemmArgs& a, int warp, int first_epi_warp, int lane) {
  epi_bar_sync();
  if (warp == first_epi_warp && lane == 0) {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    bool signal = true;
    if (a.scat_local != nullptr) {
      uint32_t old;
      asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(a.scat_local) : "memory");
      signal = old == gridDim.x - 1;
      if (signal) {
        asm volatile("st.relaxed.gpu.global.u32 [%0], 0;" ::"l"(a.scat_local) : "memory");
        asm volatile("fence.acq_rel.sys;" ::: "memory");
      }
    }
    if (signal)
      for (int q = 0; q < a.scat_nranks; ++q)
        asm volatile("red.relaxed.sys.global.add.u32 [%0], 1;" ::"l"(a.scat_count[q]) : "memory");
  }
}

// Per-role timestamps of CTA 0 and per-phase cycle totals for pipeline diagnostics; compiled in only
// with -DVMC_GEMM_TRACE=1 (the default build has no timing code in the hot loops).
#ifndef VMC_GEMM_TRACE
#define VMC_GEMM_TRACE 0
#endif
__device__ __forceinline__ void trace_at(const GemmArgs& a, int slot) {
  if constexpr (VMC_GEMM_TRACE != 0) {
    if (a.trace != nullptr && blockIdx.x == 0 && slot < 512) a.trace[slot] = clock64();
  }
}
// Diagnostic builds (-DVMC_GEMM_SKIP=mask) drop stages of the decode kernel to expose how much of
// its time each stage costs: 1 dequant arithmetic, 2 MMAs, 4 weight loads, 8 TMEM stores. The
// outputs of such builds are meaningless; the default build skips nothing. 16 leaves the kernel
// right after its set-up (the fixed cost of a launch); 32 drops the activation loads, 64 the
// epilogue's reads and stores.
#ifndef VMC_GEMM_SKIP
#define VMC_GEMM_SKIP 0
#endif

struct PhaseClock {
  long long t = 0;
  __device__ __forceinline__ void start() {
    if constexpr (VMC_GEMM_TRACE != 0) t = clock64();
  }
  __device__ __forceinline__ long long lap() {
    if constexpr (VMC_GEMM_TRACE != 0) {
      const long long n = clock64(), d = n - t;
      t = n;
      return d;
    }
    return 0;
  }
};
__device__ __forceinline__ void phase_add(const GemmArgs& a, int slot, long long v) {
  if constexpr (VMC_GEMM_TRACE != 0) {
    if (a.trace != nullptr) atomicAdd(a.trace + 768 + slot, static_cast<unsigned long long>(v));
  }
}

// Work unit u -> (group, n tile, m tile, split). m fastest: concurrently running CTAs share a weight
// tile, so in prefill the tile is fetched from HBM once and re-read from L2 by the other token
// tiles. `rows` <= 0 marks a unit past the end of its group (grouped mode); every role skips it.
struct Unit {
  int nt, mt, split, c0, c1;
  int row0;     // first row of X / of the output covered by the tile
  int rows;     // valid rows of the tile
  size_t wtile; // byte offset of the unit's first weight tile (chunk 0)
  int rot;      // the decode kernel walks chunks c0 + (i + rot) % (c1 - c0), i = 0 .. c1 - c0 - 1
  __device__ __forceinline__ int nchunks() const { return c1 - c0; }
  __device__ __forceinline__ int chunk(int i) const {
    const int n = c1 - c0;
    const int j = i + rot;
    return c0 + (j >= n ? j - n : j);
  }
};
__device__ __forceinline__ Unit unit_of(const GemmArgs& a, int u, int tile_bytes) {
  Unit r;
  int g = 0;
  if (a.groups > 0) {
    // Grouped: n fastest, then m, then group, so the (usually non-empty) first m tile of every
    // group spreads over consecutive CTAs instead of landing on every m_tiles-th one.
    r.nt = u % a.n_tiles;
    const int rest = u / a.n_tiles;
    r.mt = rest % a.m_tiles;
    g = rest / a.m_tiles;
    r.split = 0;
  } else {
    r.mt = u % a.m_tiles;
    const int rest = u / a.m_tiles;
    r.split = rest % a.splits;
    r.nt = rest / a.splits;
  }
  r.c0 = r.split * a.chunks_per_split;
  r.c1 = min(a.KC, r.c0 + a.chunks_per_split);
  r.wtile = static_cast<size_t>(r.nt) * a.KC * tile_bytes;
  if (a.groups > 0) {
    const int cnt = a.grp_count[g];
    r.row0 = a.grp_offset[g] + r.mt * a.bn;
    r.rows = min(a.bn, cnt - r.mt * a.bn);
    r.wtile += static_cast<size_t>(g) * a.grp_w_stride;
  } else {
    r.row0 = r.mt * a.bn;
    r.rows = min(a.bn, a.M - r.row0);
  }
  // Units that run at the same time start at different K chunks, so that the CTAs do not all read
  // the same activation tile from L2 at once.
  const int n = r.c1 - r.c0;
  r.rot = n > 0 ? u % n : 0;
  return r;
}

// Work enumeration of the decode kernel: round-robin units, or one stream-K chunk range per CTA.
struct UnitIter {
  int u, step;
  long long x, e;
};
__device__ __forceinline__ UnitIter iter_begin(const GemmArgs& a, int first, int step) {
  UnitIter it;
  it.u = first;
  it.step = step;
  it.x = it.e = 0;
  if (a.sk) {
    const long long W = static_cast<long long>(a.n_tiles) * a.KC;
    it.x = static_cast<long long>(blockIdx.x) * W / gridDim.x;
    it.e = static_cast<long long>(blockIdx.x + 1) * W / gridDim.x;
  }
  return it;
}
__device__ __forceinline__ bool iter_next(const GemmArgs& a, UnitIter& it, Unit& w, int tile_bytes) {
  if constexpr ((VMC_GEMM_SKIP & 16) != 0) return false;
  if (a.sk) {
    if (it.x >= it.e) return false;
    const int nt = static_cast<int>(it.x / a.KC);
    const int c0 = static_cast<int>(it.x - static_cast<long long>(nt) * a.KC);
    const int c1 = static_cast<int>(min(static_cast<long long>(a.KC), c0 + (it.e - it.x)));
    w.nt = nt;
    w.mt = 0;
    w.split = 0;
    w.c0 = c0;
    w.c1 = c1;
    w.row0 = 0;
    w.rows = min(a.bn, a.M);
    w.wtile = static_cast<size_t>(nt) * a.KC * tile_bytes;
    w.rot = 0;
    it.x += c1 - c0;
    return true;
  }
  while (it.u < a.units) {
    w = unit_of(a, it.u, tile_bytes);
    it.u += it.step;
    if (w.rows > 0) return true;
  }
  return false;
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

template <int WF, int BN>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ CUtensorMap xmap, GemmArgs args) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // Align to 1024 B (128B-swizzle atoms) by offsetting the shared pointer itself: rounding through
  // an integer would drop the shared address space and turn every ring access into a generic one.
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  constexpr GemmSmemPlan P = make_plan(WF, BN);
  constexpr int SUBS = (WF == kWfBF16) ? 1 : 4;  // 64-K substeps per chunk
  constexpr uint32_t kAccCols = BN < 32 ? 32 : BN;
  constexpr uint32_t kTmemCols = 2 * kAccCols;
  constexpr bool quant = WF != kWfBF16;
  uint8_t* sA = smem;
  uint8_t* sB = smem + P.off_b();
  uint8_t* sRaw = smem + P.off_raw();
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P.off_bar());
  uint64_t* a_full = bars;
  uint64_t* a_empty = a_full + P.a_stages;
  uint64_t* b_full = a_empty + P.a_stages;
  uint64_t* b_empty = b_full + P.b_stages;
  uint64_t* raw_full = b_empty + P.b_stages;
  uint64_t* raw_empty = raw_full + P.raw_stages;
  uint64_t* acc_full = raw_empty + P.raw_stages;  // [2]
  uint64_t* acc_empty = acc_full + 2;             // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile uint32_t* abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  pdl_trigger();
  if (threadIdx.x == 0) {
    for (int i = 0; i < P.a_stages; ++i) {
      mbar_init(&a_full[i], quant ? kDequantWarps : 1);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < P.b_stages; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    for (int i = 0; i < P.raw_stages; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], kDequantWarps);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int first = blockIdx.x, step = gridDim.x;
  // Grouped mode: the unit list depends on row counts written by the previous kernels, so every
  // role (the weight producer included) waits for them before enumerating its units.
  if (args.groups > 0) pdl_wait();

  if (warp == 0) {
    // ---------------- weight producer ----------------
    if (lane == 0) {
      // Weights are constant: the stream starts before (and never waits on) the programmatic
      // dependency, so its latency overlaps the previous kernel.
      const uint64_t pol = l2_policy_evict_first();
      int st = 0;
      uint32_t ph = 0;
      for (int u = first; u < args.units && !*abort_flag; u += step) {
        const Unit w = unit_of(args, u, wf_tile_bytes(WF));
        if (w.rows <= 0) continue;
        const uint8_t* wbase = args.w + w.wtile;
        for (int c = w.c0; c < w.c1; ++c) {
          const uint8_t* wt = wbase + static_cast<size_t>(c) * wf_tile_bytes(WF);
          if (quant) {
            if (!mbar_wait(&raw_empty[st], ph ^ 1, args.err, kErrGemmWait)) { *abort_flag = 1; break; }
            mbar_arrive_expect_tx(&raw_full[st], wf_tile_bytes(WF));
            trace_at(args, 224 + (c - w.c0));
            bulk_load_evict_first(sRaw + st * P.raw_bytes(), wt, wf_tile_bytes(WF), &raw_full[st], pol);
            if (++st == P.raw_stages) { st = 0; ph ^= 1; }
          } else {
            if (!mbar_wait(&a_empty[st], ph ^ 1, args.err, kErrGemmWait)) { *abort_flag = 1; break; }
            mbar_arrive_expect_tx(&a_full[st], P.a_bytes());
            bulk_load_evict_first(sA + st * P.a_bytes(), wt, P.a_bytes(), &a_full[st], pol);
            if (++st == P.a_stages) { st = 0; ph ^= 1; }
          }
        }
      }
    }
  } else if (warp == kBWarp) {
    // ---------------- activation producer ----------------
    if (lane == 0) {
      pdl_wait();
      int st = 0;
      uint32_t ph = 0;
      for (int u = first; u < args.units && !*abort_flag; u += step) {
        const Unit w = unit_of(args, u, wf_tile_bytes(WF));
        if (w.rows <= 0) continue;
        for (int c = w.c0; c < w.c1; ++c) {
          for (int sub = 0; sub < SUBS; ++sub) {
            if (!mbar_wait(&b_empty[st], ph ^ 1, args.err, kErrGemmWait)) { *abort_flag = 1; break; }
            mbar_arrive_expect_tx(&b_full[st], P.b_bytes());
            trace_at(args, 256 + (c - w.c0) * SUBS + sub);
            tma_load_2d(sB + st * P.b_bytes(), &xmap, &b_full[st], (c * SUBS + sub) * 64, w.row0);
            if (++st == P.b_stages) { st = 0; ph ^= 1; }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(128, BN);
      int ast = 0, bst = 0;
      uint32_t aph = 0, bph = 0;
      int acc = 0;
      uint32_t acc_ph = 0;
      for (int u = first; u < args.units && !*abort_flag; u += step) {
        const Unit w = unit_of(args, u, wf_tile_bytes(WF));
        if (w.rows <= 0) continue;
        if (!mbar_wait(&acc_empty[acc], acc_ph ^ 1, args.err, kErrGemmWait)) { *abort_flag = 1; break; }
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(acc) * kAccCols;
        const int total = (w.c1 - w.c0) * SUBS;
        for (int i = 0; i < total; ++i) {
          if (!mbar_wait(&b_full[bst], bph, args.err, kErrGemmWait)) { *abort_flag = 1; break; }
          trace_at(args, 64 + i);
          if (!mbar_wait(&a_full[ast], aph, args.err, kErrGemmWait)) { *abort_flag = 1; break; }
          trace_at(args, i);
          tc_fence_after();
          const uint64_t a0 = umma_sdesc_sw128(smem_u32(sA + ast * P.a_bytes()));
          const uint64_t b0 = umma_sdesc_sw128(smem_u32(sB + bst * P.b_bytes()));
#pragma unroll
          for (int k = 0; k < 4; ++k) umma_bf16(d, a0 + 2 * k, b0 + 2 * k, idesc, (i > 0 || k > 0) ? 1u : 0u);
          umma_commit(&a_empty[ast]);
          umma_commit(&b_empty[bst]);
          if (++ast == P.a_stages) { ast = 0; aph ^= 1; }
          if (++bst == P.b_stages) { bst = 0; bph ^= 1; }
        }
        umma_commit(&acc_full[acc]);
        if (++acc == 2) { acc = 0; acc_ph ^= 1; }
      }
    }
  } else if (warp < kFirstDqWarp + kDequantWarps) {
    // ---------------- dequant (quantized formats) ----------------
    // Each warp owns 16 rows of the tile. A stages are filled and handed to the MMA one at a time
    // (one proxy fence per 64-K stage), so the dequant of the next chunk overlaps the MMAs of the
    // current one instead of waiting for its whole chunk of stages to drain.
    if constexpr (quant) {
      static_assert(P.a_stages >= 4, "a chunk needs four A stages");
      const int t = threadIdx.x - kFirstDqWarp * 32;  // 0..255
      const int r = t >> 1, h = t & 1;
      uint32_t sw_off[4];
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) sw_off[cc] = sw128_offset(r, 4 * h + cc);
      int st = 0, rst = 0;
      uint32_t ph = 0, rph = 0;
      for (int u = first; u < args.units && !*abort_flag; u += step) {
        const Unit w = unit_of(args, u, wf_tile_bytes(WF));
        if (w.rows <= 0) continue;
        bool ok = true;
        for (int c = w.c0; c < w.c1 && ok; ++c) {
          if (!mbar_wait(&raw_full[rst], rph, args.err, kErrGemmWait)) { *abort_flag = 1; ok = false; break; }
          if (warp == kFirstDqWarp && lane == 0) trace_at(args, 128 + (c - w.c0));
          const uint8_t* row = sRaw + rst * P.raw_bytes() + r * wf_row_bytes(WF);
          Q4KChunk qc;
          if constexpr (WF == kWfQ4K) q4k_prep(row, h, qc);
#pragma unroll
          for (int sub = 0; sub < SUBS; ++sub) {
            uint32_t o[16];
            if constexpr (WF == kWfQ4K) q4k_sub(row, sub, h, qc, o);
            else if constexpr (WF == kWfQ6K) dq_q6k(row, sub, h, o);
            else dq_q8_0(row, sub, h, o);
            if (!mbar_wait(&a_empty[st], ph ^ 1, args.err, kErrGemmWait)) { *abort_flag = 1; ok = false; break; }
            uint8_t* a = sA + st * P.a_bytes();
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
              *reinterpret_cast<uint4*>(a + sw_off[cc]) = make_uint4(o[4 * cc], o[4 * cc + 1], o[4 * cc + 2], o[4 * cc + 3]);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              mbar_arrive(&a_full[st]);
              if (sub == SUBS - 1) mbar_arrive(&raw_empty[rst]);
            }
            if (++st == P.a_stages) { st = 0; ph ^= 1; }
          }
          if (!ok) break;
          if (warp == kFirstDqWarp && lane == 0) trace_at(args, 160 + (c - w.c0));
          if (++rst == P.raw_stages) { rst = 0; rph ^= 1; }
        }
        if (!ok) break;
      }
    }
  } else {
    // ---------------- epilogue (warps 11..14 -> TMEM lane quarter warp % 4) ----------------
    pdl_wait();  // outputs may still be read by the previous kernel
    const int q = warp & 3;
    const int n_local = 32 * q + lane;
    int acc = 0;
    uint32_t acc_ph = 0;
    for (int u = first; u < args.units && !*abort_flag; u += step) {
      const Unit w = unit_of(args, u, wf_tile_bytes(WF));
        if (w.rows <= 0) continue;
      if (!mbar_wait(&acc_full[acc], acc_ph, args.err, kErrGemmWait)) { *abort_flag = 1; break; }
      tc_fence_after();
      const uint32_t d = tmem + static_cast<uint32_t>(acc) * kAccCols + (static_cast<uint32_t>(32 * q) << 16);
      float* outf = reinterpret_cast<float*>(args.out);
      if (args.out_mode == kGemmOutF32Split) outf += w.split * args.split_stride;
      for (int cb = 0; cb < BN; cb += 16) {
        uint32_t v[16];
        tmem_ld16(d + static_cast<uint32_t>(cb), v);
        tmem_ld_wait();
        const int m_base = w.row0 + cb;
        const int m_end = w.row0 + w.rows;
        if (args.out_mode == kGemmOutSwiGLU) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float mine = __uint_as_float(v[j]);
            const float other = __shfl_xor_sync(0xffffffffu, mine, 1);
            const int m = m_base + j;
            if ((lane & 1) == 0 && m < m_end) {
              const float y = __fdividef(mine, 1.f + __expf(-mine)) * other;
              const int f = w.nt * 64 + (n_local >> 1);
              if (f < args.N / 2)
                reinterpret_cast<__nv_bfloat16*>(args.out)[static_cast<size_t>(m) * args.ldo + f] = __float2bfloat16(y);
            }
          }
        } else if (args.out_mode == kGemmOutScatterBF16) {
          const int n = w.nt * 128 + n_local;
          if (n < args.N) scatter_rows(args, w.split, n, m_base, m_end, v);
        } else if (args.out_mode == kGemmOutRowScatterBF16) {
          const int n = w.nt * 128 + n_local;
          if (n < args.N) row_scatter_rows(args, n, m_base, m_end, v);
        } else {
          const int n = w.nt * 128 + n_local;
          if (n < args.N) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int m = m_base + j;
              if (m < m_end) {
                const float y = __uint_as_float(v[j]);
                const size_t idx = static_cast<size_t>(m) * args.ldo + n;
                if (args.out_mode == kGemmOutF32Add) atomicAdd(outf + idx, y);
                else if (args.out_mode == kGemmOutBF16) reinterpret_cast<__nv_bfloat16*>(args.out)[idx] = __float2bfloat16(y);
                else outf[idx] = y;
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
      if (++acc == 2) { acc = 0; acc_ph ^= 1; }
    }
    if (args.out_mode == kGemmOutScatterBF16 || args.out_mode == kGemmOutRowScatterBF16)
      scatter_release(args, warp, kFirstEpiWarp, lane);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------------------------
// Decode-width tiles (BN <= 64): dequantised A operand in TMEM, two independent substep groups.
//
// With both operands in shared memory every 256-K chunk moves ~230 KB through the SM's shared
// memory (raw tile in and out, bf16 A written by the dequant warps and read by the MMA, activation
// tile in and out), more than the chunk's HBM bytes take to arrive. Here the dequant warps write
// the bf16 A operand straight into TMEM (tcgen05.st) and the MMA reads it from there
// (tcgen05.mma with A in tensor memory), which removes the 128 KB of A traffic.
//
// Measured on B200: a 128xNx16 MMA with N <= 64 takes ~45 cycles, and each mbarrier wait or
// commit in an issuing thread's loop stalls its issue stream for about as long, so a pipeline in
// which one MMA thread waits for all dequant warps (and they for it) leaves the tensor pipe idle.
// The 16 dequant warps therefore form two groups; group G owns K substeps 2G and 2G+1 (128 K) of
// every chunk, writes them into its own TMEM A slots (two, so the dequant runs a chunk ahead of the
// MMA) and has its own MMA-issuing warp accumulating into its own TMEM accumulator;
// the epilogue adds the two. One group's handshakes overlap the other group's MMAs. Accumulators
// are double-buffered per group, so a unit's epilogue (measured at ~5 us for the SwiGLU output of
// a 128-row unit while the dequant warps share the SM) overlaps the next unit's MMAs.
// TMEM: accumulators [0, 256) (buffer b, group G at (2b + G) * 64), A slots [256, 512)
// (64 columns = 128 K each).
//
// Warp roles in a 768-thread CTA:
//   warp 0       weight producer (raw ring, one cp.async.bulk per tile) and TMEM allocation
//   warp 1       activation producer (one chunk-wide stage = 4 TMA boxes)
//   warps 2, 3   MMA issuers of groups 0, 1
//   warps 4-19   dequant: group (w - 4) / 8, substep 2 * group + ((w - 4) / 4) % 2, lane quarter w % 4
//   warps 20-23  epilogue (lane quarter w % 4)

constexpr int kDThreads = 768;
constexpr int kDFirstDq = 4;
constexpr int kDFirstEpi = 20;
constexpr int kDSlots = 2;
constexpr uint32_t kDACol = 256;

// 64 K-values of substep S of one Q4_K row: o[0..15] = sub-block 2S, o[16..31] = sub-block 2S + 1
// (bf16 pairs in K order). Per 8 values: 3 shifts + 4 lop3 on the integer pipe, 4 sub + 4 fma.
template <int S>
__device__ __forceinline__ void q4k_row64(const uint8_t* row, uint32_t (&o)[32]) {
  const uint2 sc = *reinterpret_cast<const uint2*>(row + 8 * S);  // (ds, ndm) of sub-blocks 2S, 2S + 1
  const uint32_t ds_lo = __byte_perm(sc.x, 0u, 0x1010), dm_lo = __byte_perm(sc.x, 0u, 0x3232);
  const uint32_t ds_hi = __byte_perm(sc.y, 0u, 0x1010), dm_hi = __byte_perm(sc.y, 0u, 0x3232);
  const uint4* q = reinterpret_cast<const uint4*>(row + 32 + 32 * S);
  const uint4 w0 = q[0], w1 = q[1];
  const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t a = lop_and_or(w[i], 0x000f000fu, kMagic128x2);
    const uint32_t b = lop_and_or(w[i] >> 8, 0x000f000fu, kMagic128x2);
    const uint32_t c = lop_and_or(w[i] >> 4, 0x000f000fu, kMagic128x2);
    const uint32_t e = lop_and_or(w[i] >> 12, 0x000f000fu, kMagic128x2);
    o[2 * i] = bfma2(bsub2(a, kMagic128x2), ds_lo, dm_lo);
    o[2 * i + 1] = bfma2(bsub2(b, kMagic128x2), ds_lo, dm_lo);
    o[16 + 2 * i] = bfma2(bsub2(c, kMagic128x2), ds_hi, dm_hi);
    o[16 + 2 * i + 1] = bfma2(bsub2(e, kMagic128x2), ds_hi, dm_hi);
  }
}

// 64 K-values of substep s (0..3, warp-uniform) of one row of a quantized tile.
template <int WF>
__device__ __forceinline__ void dq_row64(const uint8_t* row, int s, uint32_t (&o)[32]) {
  if constexpr (WF == kWfQ4K) {
    switch (s) {
      case 0: q4k_row64<0>(row, o); break;
      case 1: q4k_row64<1>(row, o); break;
      case 2: q4k_row64<2>(row, o); break;
      default: q4k_row64<3>(row, o); break;
    }
  } else {
    uint32_t (&lo)[16] = *reinterpret_cast<uint32_t(*)[16]>(&o[0]);
    uint32_t (&hi)[16] = *reinterpret_cast<uint32_t(*)[16]>(&o[16]);
    if constexpr (WF == kWfQ6K) {
      dq_q6k(row, s, 0, lo);
      dq_q6k(row, s, 1, hi);
    } else {
      dq_q8_0(row, s, 0, lo);
      dq_q8_0(row, s, 1, hi);
    }
  }
}

struct GemmDPlan {
  int b_stages = 0;
  int raw_stages = 0;
  int bn = 0;
  int wf = 0;
  __host__ __device__ constexpr int b_box() const { return bn * 128; }
  __host__ __device__ constexpr int b_bytes() const { return 4 * b_box(); }
  __host__ __device__ constexpr int raw_bytes() const { return wf_tile_bytes(wf); }
  __host__ __device__ constexpr int off_raw() const { return b_stages * b_bytes(); }
  __host__ __device__ constexpr int off_bar() const { return off_raw() + raw_stages * raw_bytes(); }
  // a_full[2 * kDSlots], slot_free[2 * kDSlots], acc_full[4], acc_empty[2], b_full/b_empty,
  // raw_full/raw_empty
  __host__ __device__ constexpr int nbars() const { return 4 * kDSlots + 6 + 2 * b_stages + 2 * raw_stages; }
  __host__ __device__ constexpr int total() const { return off_bar() + nbars() * 8 + 16 + 1024; }
};

// Activation stages first (a chunk-wide stage is read by both groups, which may be a chunk apart),
// then raw weight stages for HBM latency.
__host__ __device__ constexpr GemmDPlan make_dplan(int wf, int bn) {
  GemmDPlan p;
  p.bn = bn;
  p.wf = wf;
  const int budget = 222 * 1024;
  p.b_stages = 2;
  p.raw_stages = 2;
  while (p.b_stages < 4) {
    GemmDPlan q = p;
    q.b_stages += 1;
    if (q.total() > budget) break;
    p = q;
  }
  while (p.raw_stages < 8) {
    GemmDPlan q = p;
    q.raw_stages += 1;
    if (q.total() > budget) break;
    p = q;
  }
  return p;
}

template <int WF, int BN>
__global__ void __launch_bounds__(kDThreads, 1) gemm_qd_kernel(const __grid_constant__ CUtensorMap xmap, GemmArgs args) {
  static_assert(BN <= 64, "decode-width kernel");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  constexpr GemmDPlan P = make_dplan(WF, BN);
  constexpr uint32_t kAccCols = BN < 32 ? 32 : BN;
  static_assert(4 * kAccCols <= kDACol && kDACol + 2 * kDSlots * 64 <= 512, "TMEM plan");
  uint8_t* sB = smem;
  uint8_t* sRaw = smem + P.off_raw();
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P.off_bar());
  uint64_t* a_full = bars;                       // [group * kDSlots + slot], 8 dequant-warp arrivals
  uint64_t* slot_free = a_full + 2 * kDSlots;    // [group * kDSlots + slot], MMA commit
  uint64_t* acc_full = slot_free + 2 * kDSlots;  // [buffer * 2 + group], MMA commit at the end of a unit
  uint64_t* acc_empty = acc_full + 4;            // [buffer], 4 epilogue-warp arrivals
  uint64_t* b_full = acc_empty + 2;
  uint64_t* b_empty = b_full + P.b_stages;       // one commit per group
  uint64_t* raw_full = b_empty + P.b_stages;
  uint64_t* raw_empty = raw_full + P.raw_stages;  // 16 dequant-warp arrivals
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(raw_empty + P.raw_stages);
  volatile uint32_t* abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  pdl_trigger();
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2 * kDSlots; ++i) {
      mbar_init(&a_full[i], 8);
      mbar_init(&slot_free[i], 1);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&acc_full[i], 1);
    for (int i = 0; i < 2; ++i) mbar_init(&acc_empty[i], 4);
    for (int i = 0; i < P.b_stages; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 2);
    }
    for (int i = 0; i < P.raw_stages; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], 16);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int first = (VMC_GEMM_SKIP & 16) != 0 ? args.units : static_cast<int>(blockIdx.x), step = gridDim.x;
  // Grouped mode: the unit list depends on row counts written by the previous kernels, so every
  // role (the weight producer included) waits for them before enumerating its units.
  if (args.groups > 0) pdl_wait();

  if (warp == 0) {
    // ---------------- weight producer (weights are constant: starts before the PDL wait) -------
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      int st = 0;
      uint32_t ph = 0;
      UnitIter it = iter_begin(args, first, step);
      Unit w;
      while (!*abort_flag && iter_next(args, it, w, wf_tile_bytes(WF))) {
        const uint8_t* wbase = args.w + w.wtile;
        for (int i = 0; i < w.nchunks(); ++i) {
          const int c = w.chunk(i);
          if (!mbar_wait(&raw_empty[st], ph ^ 1, args.err, kErrGemmWait)) { *abort_flag = 1; break; }
          if constexpr ((VMC_GEMM_SKIP & 4) != 0) {
            mbar_arrive(&raw_full[st]);
          } else {
            mbar_arrive_expect_tx(&raw_full[st], wf_tile_bytes(WF));
            bulk_load_evict_first(sRaw + st * P.raw_bytes(), wbase + static_cast<size_t>(c) * wf_tile_bytes(WF),
                                  wf_tile_bytes(WF), &raw_full[st], pol);
          }
          if (++st == P.raw_stages) { st = 0; ph ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- activation producer ----------------
    if (lane == 0) {
      pdl_wait();
      int st = 0;
      uint32_t ph = 0;
      UnitIter it = iter_begin(args, first, step);
      Unit w;
      while (!*abort_flag && iter_next(args, it, w, wf_tile_bytes(WF))) {
        for (int i = 0; i < w.nchunks(); ++i) {
          const int c = w.chunk(i);
          if (!mbar_wait(&b_empty[st], ph ^ 1, args.err, kErrGemmWait)) { *abort_flag = 1; break; }
          if constexpr ((VMC_GEMM_SKIP & 32) != 0) {
            mbar_arrive(&b_full[st]);
          } else {
            mbar_arrive_expect_tx(&b_full[st], P.b_bytes());
#pragma unroll
            for (int i = 0; i < 4; ++i)
              tma_load_2d(sB + st * P.b_bytes() + i * P.b_box(), &xmap, &b_full[st], (c * 4 + i) * 64, w.row0);
          }
          if (++st == P.b_stages) { st = 0; ph ^= 1; }
        }
      }
    }
  } else if (warp == 2 || warp == 3) {
    // ---------------- MMA issuer of group G ----------------
    if (lane == 0) {
      const int G = warp - 2;
      constexpr uint32_t idesc = umma_idesc_bf16(128, BN);
      int g = 0;   // CTA-wide chunk counter
      int ui = 0;  // units of this CTA so far: accumulator buffer ui & 1
      bool ok = true;
      PhaseClock pc;
      long long ph_acc = 0, ph_a = 0, ph_b = 0, ph_mma = 0;
      pc.start();
      UnitIter it = iter_begin(args, first, step);
      Unit w;
      while (ok && !*abort_flag && iter_next(args, it, w, wf_tile_bytes(WF))) {
        const int buf = ui & 1;
        if (!mbar_wait(&acc_empty[buf], ((ui >> 1) & 1) ^ 1, args.err, kErrGemmWait)) { ok = false; break; }
        ph_acc += pc.lap();
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(2 * buf + G) * kAccCols;
        for (int i = 0; i < w.nchunks(); ++i, ++g) {
          const int k = g % kDSlots;
          const int bst = g % P.b_stages;
          ph_mma += pc.lap();
          if (!mbar_wait(&a_full[G * kDSlots + k], (g / kDSlots) & 1, args.err, kErrGemmWait)) { ok = false; break; }
          ph_a += pc.lap();
          if (!mbar_wait(&b_full[bst], (g / P.b_stages) & 1, args.err, kErrGemmWait)) { ok = false; break; }
          ph_b += pc.lap();
          tc_fence_after();
          const uint32_t a0 = tmem + kDACol + static_cast<uint32_t>(G * kDSlots + k) * 64;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint64_t b0 = umma_sdesc_sw128(smem_u32(sB + bst * P.b_bytes() + (2 * G + h) * P.b_box()));
#pragma unroll
            for (int k4 = 0; k4 < 4; ++k4)
              if constexpr ((VMC_GEMM_SKIP & 2) == 0)
                umma_bf16_ts(d, a0 + h * 32 + 8 * k4, b0 + 2 * k4, idesc, (i > 0 || h > 0 || k4 > 0) ? 1u : 0u);
          }
          umma_commit(&slot_free[G * kDSlots + k]);
          umma_commit(&b_empty[bst]);
        }
        if (!ok) break;
        umma_commit(&acc_full[2 * buf + G]);
        ++ui;
      }
      if (!ok) *abort_flag = 1;
      ph_mma += pc.lap();
      phase_add(args, 8, ph_acc);
      phase_add(args, 9, ph_a);
      phase_add(args, 10, ph_b);
      phase_add(args, 11, ph_mma);
      phase_add(args, 12, g);
    }
  } else if (warp >= kDFirstDq && warp < kDFirstEpi) {
    // ---------------- dequant -> TMEM ----------------
    const int q = warp & 3;
    const int G = (warp - kDFirstDq) >> 3;
    const int h = ((warp - kDFirstDq) >> 2) & 1;
    const int s = 2 * G + h;  // K substep of this warp
    const uint32_t lane_base = static_cast<uint32_t>(32 * q) << 16;
    int rst = 0;
    uint32_t rph = 0;
    int g = 0;
    PhaseClock pc;
    long long ph_raw = 0, ph_dq = 0, ph_slot = 0, ph_st = 0, ph_rest = 0;
    pc.start();
    UnitIter it = iter_begin(args, first, step);
    Unit w;
    while (!*abort_flag && iter_next(args, it, w, wf_tile_bytes(WF))) {
      bool ok = true;
      for (int i = 0; i < w.nchunks(); ++i, ++g) {
        ph_rest += pc.lap();
        if (!mbar_wait(&raw_full[rst], rph, args.err, kErrGemmWait)) { ok = false; break; }
        ph_raw += pc.lap();
        const uint8_t* row = sRaw + rst * P.raw_bytes() + (32 * q + lane) * wf_row_bytes(WF);
        uint32_t o[32];
        if constexpr ((VMC_GEMM_SKIP & 1) != 0) {
          const uint4* r4 = reinterpret_cast<const uint4*>(row);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint4 v = r4[i & 3];
            o[4 * i] = v.x; o[4 * i + 1] = v.y; o[4 * i + 2] = v.z; o[4 * i + 3] = v.w;
          }
        } else {
          dq_row64<WF>(row, s, o);
        }
        __syncwarp();
        ph_dq += pc.lap();
        if (lane == 0) mbar_arrive(&raw_empty[rst]);
        const int k = g % kDSlots;
        if (!mbar_wait(&slot_free[G * kDSlots + k], ((g / kDSlots) & 1) ^ 1, args.err, kErrGemmWait)) { ok = false; break; }
        ph_slot += pc.lap();
        tc_fence_after();
        const uint32_t ta = tmem + lane_base + kDACol + static_cast<uint32_t>(G * kDSlots + k) * 64 + h * 32;
        if constexpr ((VMC_GEMM_SKIP & 8) == 0) {
          tmem_st16(ta, o);
          tmem_st16(ta + 16, o + 16);
          tmem_st_wait();
        } else {
          if (o[0] == 0x7fffffffu && o[31] == 0x7fffffffu) args.err[0] = o[7];  // keeps the loads live
        }
        tc_fence_before();
        __syncwarp();
        ph_st += pc.lap();
        if (lane == 0) mbar_arrive(&a_full[G * kDSlots + k]);
        if (++rst == P.raw_stages) { rst = 0; rph ^= 1; }
      }
      if (!ok) { *abort_flag = 1; break; }
    }
    if (lane == 0) {
      phase_add(args, 0, ph_raw);
      phase_add(args, 1, ph_dq);
      phase_add(args, 2, ph_slot);
      phase_add(args, 3, ph_st);
      phase_add(args, 4, ph_rest);
      phase_add(args, 5, g);
    }
  } else if (warp >= kDFirstEpi && warp < kDFirstEpi + 4) {
    // ---------------- epilogue: sum of the two group accumulators ----------------
    pdl_wait();  // outputs may still be read by the previous kernel
    const int q = warp & 3;
    const int n_local = 32 * q + lane;
    int ui = 0;
    PhaseClock pc;
    long long ph_ew = 0, ph_ld = 0, ph_out = 0;
    pc.start();
    UnitIter it = iter_begin(args, first, step);
    Unit w;
    while (!*abort_flag && iter_next(args, it, w, wf_tile_bytes(WF))) {
      const int buf = ui & 1;
      const uint32_t acc_ph = (ui >> 1) & 1;
      const bool ok = mbar_wait(&acc_full[2 * buf], acc_ph, args.err, kErrGemmWait) &&
                      mbar_wait(&acc_full[2 * buf + 1], acc_ph, args.err, kErrGemmWait);
      if (!ok) { *abort_flag = 1; break; }
      // Stream-K: a segment after chunk 0 of its tile stores a partial; the segment holding chunk 0
      // of a split tile first waits for the later CTAs' partials.
      const bool sk_part = args.sk && w.c0 > 0;
      const bool sk_head = args.sk && w.c0 == 0 && w.c1 < args.KC;
      int n_contrib = 0;
      if (sk_head) {
        const long long W = static_cast<long long>(args.n_tiles) * args.KC, G = gridDim.x;
        const long long xlast = static_cast<long long>(w.nt + 1) * args.KC - 1;
        n_contrib = static_cast<int>(((xlast + 1) * G + W - 1) / W - 1) - static_cast<int>(blockIdx.x);
        int good = 1;
        if (lane == 0) {
          const long long t0 = clock64();
          while (static_cast<int>(ld_acquire_gpu(args.sk_cnt + w.nt)) < n_contrib) {
            if (clock64() - t0 > (4ll << 30)) {
              atomicCAS(args.err, 0u, static_cast<uint32_t>(kErrGemmWait));
              good = 0;
              break;
            }
          }
        }
        good = __shfl_sync(0xffffffffu, good, 0);
        if (!good) { *abort_flag = 1; break; }
      }
      ph_ew += pc.lap();
      tc_fence_after();
      const uint32_t d = tmem + static_cast<uint32_t>(2 * buf) * kAccCols + (static_cast<uint32_t>(32 * q) << 16);
      float* outf = reinterpret_cast<float*>(args.out);
      if (args.out_mode == kGemmOutF32Split) outf += w.split * args.split_stride;
#pragma unroll 1
      for (int cb = 0; cb < ((VMC_GEMM_SKIP & 64) != 0 ? 0 : BN); cb += 16) {
        uint32_t v[16], t[16];
        tmem_ld16(d + static_cast<uint32_t>(cb), v);
        tmem_ld16(d + kAccCols + static_cast<uint32_t>(cb), t);
        tmem_ld_wait();
        ph_ld += pc.lap();
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) + __uint_as_float(t[j]));
        if (sk_part) {
          float* slot = args.sk_ws + static_cast<size_t>(blockIdx.x) * (BN * 128);
#pragma unroll
          for (int j = 0; j < 16; ++j) slot[(cb + j) * 128 + n_local] = __uint_as_float(v[j]);
          continue;
        }
        for (int c = 1; c <= n_contrib; ++c) {
          const float* slot = args.sk_ws + static_cast<size_t>(blockIdx.x + c) * (BN * 128);
#pragma unroll
          for (int j = 0; j < 16; ++j)
            v[j] = __float_as_uint(__uint_as_float(v[j]) + __ldcg(slot + (cb + j) * 128 + n_local));
        }
        const int m_base = w.row0 + cb;
        const int m_end = w.row0 + w.rows;
        if (args.out_mode == kGemmOutSwiGLU) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float mine = __uint_as_float(v[j]);
            const float other = __shfl_xor_sync(0xffffffffu, mine, 1);
            const int m = m_base + j;
            if ((lane & 1) == 0 && m < m_end) {
              const float y = __fdividef(mine, 1.f + __expf(-mine)) * other;
              const int f = w.nt * 64 + (n_local >> 1);
              if (f < args.N / 2)
                reinterpret_cast<__nv_bfloat16*>(args.out)[static_cast<size_t>(m) * args.ldo + f] = __float2bfloat16(y);
            }
          }
        } else if (args.out_mode == kGemmOutScatterBF16) {
          const int nn = w.nt * 128 + n_local;
          if (nn < args.N) scatter_rows(args, w.split, nn, m_base, m_end, v);
        } else if (args.out_mode == kGemmOutRowScatterBF16) {
          const int nn = w.nt * 128 + n_local;
          if (nn < args.N) row_scatter_rows(args, nn, m_base, m_end, v);
        } else {
          const int nn = w.nt * 128 + n_local;
          if (nn < args.N) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int m = m_base + j;
              if (m < m_end) {
                const float y = __uint_as_float(v[j]);
                const size_t idx = static_cast<size_t>(m) * args.ldo + nn;
                if (args.out_mode == kGemmOutF32Add) atomicAdd(outf + idx, y);
                else if (args.out_mode == kGemmOutBF16) reinterpret_cast<__nv_bfloat16*>(args.out)[idx] = __float2bfloat16(y);
                else outf[idx] = y;
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      ++ui;
      if (sk_part || sk_head) {
        epi_bar_sync();  // all four epilogue warps have stored (partial) or read (finisher) the slots
        if (warp == kDFirstEpi && lane == 0) {
          if (sk_part) {
            __threadfence();
            atomicAdd(args.sk_cnt + w.nt, 1u);
          } else {
            args.sk_cnt[w.nt] = 0;  // every contributor has counted: ready for the next launch
          }
        }
      }
      ph_out += pc.lap();
    }
    if (lane == 0) {
      phase_add(args, 13, ph_ew);
      phase_add(args, 14, ph_ld);
      phase_add(args, 15, ph_out);
    }
    if (args.out_mode == kGemmOutScatterBF16 || args.out_mode == kGemmOutRowScatterBF16)
      scatter_release(args, warp, kDFirstEpi, lane);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------------------------
// Host side

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    VMC_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    VMC_CHECK(p != nullptr && q == cudaDriverEntryPointSuccess, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    VMC_CUDA_CHECK(cudaGetDevice(&dev));
    VMC_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  }
  return n;
}

template <int WF, int BN>
int launch(const CUtensorMap& map, const GemmArgs& a, cudaStream_t st) {
  constexpr GemmSmemPlan P = make_plan(WF, BN);
  static_assert(P.total() <= 227 * 1024, "shared memory plan too large");
  static bool configured = false;
  if (!configured) {
    VMC_CUDA_CHECK(cudaFuncSetAttribute(gemm_kernel<WF, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, P.total()));
    configured = true;
  }
  const int grid = a.units < num_sms() ? a.units : num_sms();
  launch_k(gemm_kernel<WF, BN>, dim3(grid), dim3(kThreads), P.total(), st, map, a);
  return grid;
}

template <int WF, int BN>
int launch_qd(const CUtensorMap& map, const GemmArgs& a, cudaStream_t st) {
  constexpr GemmDPlan P = make_dplan(WF, BN);
  static_assert(P.total() <= 227 * 1024, "shared memory plan too large");
  // More than half the SM's shared memory: no second CTA (and no second 512-column TMEM
  // allocation) can be resident on the SM.
  static_assert(P.total() > 114 * 1024, "the TMEM plan assumes one CTA per SM");
  static bool configured = false;
  if (!configured) {
    VMC_CUDA_CHECK(cudaFuncSetAttribute(gemm_qd_kernel<WF, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, P.total()));
    configured = true;
  }
  const int grid = a.units < num_sms() ? a.units : num_sms();
  launch_k(gemm_qd_kernel<WF, BN>, dim3(grid), dim3(kDThreads), P.total(), st, map, a);
  return grid;
}

// Quantized weights with decode-width token tiles take the TMEM-A kernel; bf16 weights and wide
// (prefill) tiles the shared-memory kernel.
template <int WF, int BN>
int launch_any(const CUtensorMap& map, const GemmArgs& a, cudaStream_t st) {
  if constexpr (WF != kWfBF16 && BN <= 64) return launch_qd<WF, BN>(map, a, st);
  else return launch<WF, BN>(map, a, st);
}

template <int WF>
int dispatch_bn(int bn, const CUtensorMap& map, const GemmArgs& a, cudaStream_t st) {
  switch (bn) {
    case 16: return launch_any<WF, 16>(map, a, st);
    case 32: return launch_any<WF, 32>(map, a, st);
    case 64: return launch_any<WF, 64>(map, a, st);
    case 128: return launch_any<WF, 128>(map, a, st);
    case 256: return launch_any<WF, 256>(map, a, st);
    default: throw std::runtime_error("gemm: unsupported BN");
  }
}

int dispatch_wf(int wf, int bn, const CUtensorMap& map, const GemmArgs& a, cudaStream_t st) {
  switch (wf) {
    case kWfBF16: return dispatch_bn<kWfBF16>(bn, map, a, st);
    case kWfQ4K: return dispatch_bn<kWfQ4K>(bn, map, a, st);
    case kWfQ6K: return dispatch_bn<kWfQ6K>(bn, map, a, st);
    case kWfQ8_0: return dispatch_bn<kWfQ8_0>(bn, map, a, st);
    default: throw std::runtime_error("gemm: unknown weight format");
  }
}

}  // namespace

void make_act_tensor_map(CUtensorMap* map, const void* x, int M, int K, int ldx, int box_rows) {
  VMC_CHECK(reinterpret_cast<uintptr_t>(x) % 16 == 0, "gemm: activation pointer must be 16-byte aligned");
  VMC_CHECK((ldx * 2) % 16 == 0, "gemm: activation row stride must be a multiple of 16 bytes");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldx) * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  VMC_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed for the activation map");
}

unsigned long long* g_gemm_trace = nullptr;
void gemm_set_trace(unsigned long long* buf) { g_gemm_trace = buf; }

int gemm_pick_bn(int M) {
  if (M <= 16) return 16;
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  if (M <= 128) return 128;
  return 256;
}

namespace {
// Stream-K workspace of the current device: partial slots for every CTA at the widest decode tile
// and one arrival counter per weight tile (zeroed once; finishers reset their counters).
constexpr int kSkMaxTiles = 1 << 14;
struct SkWorkspace {
  float* ws = nullptr;
  uint32_t* cnt = nullptr;
};
SkWorkspace g_sk[64];

bool streamk_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("VMC_STREAMK");
    return !(e && std::strcmp(e, "0") == 0);
  }();
  return on;
}

SkWorkspace& sk_workspace() {
  int dev = 0;
  VMC_CUDA_CHECK(cudaGetDevice(&dev));
  SkWorkspace& w = g_sk[dev];
  if (!w.ws) {
    VMC_CUDA_CHECK(cudaMalloc(&w.ws, static_cast<size_t>(num_sms()) * 64 * 128 * sizeof(float)));
    VMC_CUDA_CHECK(cudaMalloc(&w.cnt, kSkMaxTiles * sizeof(uint32_t)));
    VMC_CUDA_CHECK(cudaMemset(w.cnt, 0, kSkMaxTiles * sizeof(uint32_t)));
  }
  return w;
}

// Decode-width quantized GEMMs with one token tile and no K split take the stream-K schedule.
bool use_streamk(int wf, int bn, int m_tiles, int splits, int n_tiles) {
  return streamk_enabled() && wf != kWfBF16 && bn <= 64 && m_tiles == 1 && splits == 1 && n_tiles <= kSkMaxTiles;
}

void apply_streamk(GemmArgs& a, cudaStream_t st) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  VMC_CUDA_CHECK(cudaStreamIsCapturing(st, &cs));
  int dev = 0;
  VMC_CUDA_CHECK(cudaGetDevice(&dev));
  VMC_CHECK(g_sk[dev].ws != nullptr || cs == cudaStreamCaptureStatusNone,
            "gemm: the stream-K workspace must be allocated (gemm_prepare) before stream capture");
  SkWorkspace& ws = sk_workspace();
  a.sk = 1;
  a.sk_ws = ws.ws;
  a.sk_cnt = ws.cnt;
  const long long W = static_cast<long long>(a.n_tiles) * a.KC;
  a.units = static_cast<int>(W < num_sms() ? W : num_sms());  // grid size: one CTA per SM at most
}

GemmArgs dense_args(int wf, const void* w_tiled, int N, int K, int M, void* out, int ldo, int out_mode, int& splits,
                    int bn, uint32_t* err, int64_t split_stride) {
  const int chunk = wf_chunk(wf);
  const int KC = (K + chunk - 1) / chunk;
  if (splits < 1) splits = 1;
  if (splits > KC) splits = KC;
  GemmArgs a = {};
  a.w = static_cast<const uint8_t*>(w_tiled);
  a.N = N;
  a.K = K;
  a.M = M;
  a.KC = KC;
  a.chunks_per_split = (KC + splits - 1) / splits;
  splits = (KC + a.chunks_per_split - 1) / a.chunks_per_split;
  a.splits = splits;
  a.n_tiles = (N + 127) / 128;
  a.m_tiles = (M + bn - 1) / bn;
  a.units = a.n_tiles * a.m_tiles * splits;
  a.out = out;
  a.ldo = ldo;
  a.out_mode = out_mode;
  a.split_stride = split_stride;
  a.err = err;
  a.trace = g_gemm_trace;
  a.bn = bn;
  a.groups = 0;
  return a;
}
}  // namespace

int gemm_tcgen05(int wf, const void* w_tiled, int N, int K, const void* x, int M, int ldx, void* out, int ldo,
                 int out_mode, int splits, int bn, uint32_t* err, cudaStream_t st, int64_t split_stride) {
  VMC_CHECK(M > 0 && N > 0 && K > 0, "gemm: empty problem");
  VMC_CHECK(out_mode != kGemmOutScatterBF16, "gemm: the scatter output mode goes through gemm_tcgen05_scatter");
  if (bn <= 0) bn = gemm_pick_bn(M);
  GemmArgs a = dense_args(wf, w_tiled, N, K, M, out, ldo, out_mode, splits, bn, err, split_stride);
  VMC_CHECK(splits == 1 || out_mode == kGemmOutF32Add || out_mode == kGemmOutF32Split,
            "gemm: split-K needs an fp32 accumulate / per-split output mode");
  if (use_streamk(wf, bn, a.m_tiles, splits, a.n_tiles)) apply_streamk(a, st);
  CUtensorMap map;
  make_act_tensor_map(&map, x, M, K, ldx, bn);
  return dispatch_wf(wf, bn, map, a, st);
}

int gemm_tcgen05_scatter(int wf, const void* w_tiled, int N, int K, const void* x, int M, int ldx, int splits,
                         void* const* recv, uint32_t* const* counters, int nranks, int rank, int64_t recv_rows,
                         uint32_t* err, cudaStream_t st, int* splits_used, uint32_t* local_count) {
  VMC_CHECK(M > 0 && N > 0 && K > 0, "gemm_scatter: empty problem");
  VMC_CHECK(nranks >= 1 && nranks <= 8 && rank >= 0 && rank < nranks, "gemm_scatter: bad ranks");
  const int bn = gemm_pick_bn(M);
  GemmArgs a = dense_args(wf, w_tiled, N, K, M, nullptr, N, kGemmOutScatterBF16, splits, bn, err, 0);
  const int rpr = (M + nranks - 1) / nranks;
  VMC_CHECK(static_cast<int64_t>(nranks) * splits * rpr <= recv_rows, "gemm_scatter: receive buffer too small");
  for (int q = 0; q < 8; ++q) {
    a.scat[q] = q < nranks ? recv[q] : nullptr;
    a.scat_count[q] = q < nranks ? counters[q] : nullptr;
  }
  a.scat_rpr = rpr;
  a.scat_rank = rank;
  a.scat_nranks = nranks;
  a.scat_local = local_count;
  if (splits_used) *splits_used = splits;
  if (use_streamk(wf, bn, a.m_tiles, splits, a.n_tiles)) apply_streamk(a, st);
  CUtensorMap map;
  make_act_tensor_map(&map, x, M, K, ldx, bn);
  return dispatch_wf(wf, bn, map, a, st);
}

void gemm_tcgen05_grouped(int wf, const void* w_tiled, int64_t w_group_stride, int N, int K, const void* x,
                          int rows_total, int ldx, void* out, int ldo, int out_mode, int groups,
                          const int32_t* counts, const int32_t* offsets, int max_rows, int bn, uint32_t* err,
                          cudaStream_t st) {
  VMC_CHECK(rows_total > 0 && N > 0 && K > 0 && groups > 0 && max_rows > 0, "gemm_grouped: empty problem");
  VMC_CHECK(out_mode == kGemmOutBF16 || out_mode == kGemmOutF32 || out_mode == kGemmOutSwiGLU,
            "gemm_grouped: bf16, fp32 or SwiGLU output");
  if (bn <= 0) bn = gemm_pick_bn(max_rows);
  const int chunk = wf_chunk(wf);
  GemmArgs a = {};
  a.w = static_cast<const uint8_t*>(w_tiled);
  a.N = N;
  a.K = K;
  a.M = rows_total;
  a.KC = (K + chunk - 1) / chunk;
  a.chunks_per_split = a.KC;
  a.splits = 1;
  a.n_tiles = (N + 127) / 128;
  a.m_tiles = (max_rows + bn - 1) / bn;
  a.units = groups * a.n_tiles * a.m_tiles;
  a.out = out;
  a.ldo = ldo;
  a.out_mode = out_mode;
  a.split_stride = 0;
  a.err = err;
  a.trace = g_gemm_trace;
  a.bn = bn;
  a.groups = groups;
  a.grp_count = counts;
  a.grp_offset = offsets;
  a.grp_w_stride = w_group_stride;
  CUtensorMap map;
  make_act_tensor_map(&map, x, rows_total, K, ldx, bn);
  dispatch_wf(wf, bn, map, a, st);
}


void gemm_prepare() { (void)sk_workspace(); }
bool gemm_streamk() { return streamk_enabled(); }

int gemm_tcgen05_grouped_rowscatter(int wf, const void* w_tiled, int64_t w_group_stride, int N, int K, const void* x,
                                    int rows_total, int ldx, int groups, const int32_t* counts, const int32_t* offsets,
                                    int max_rows, int bn, const int32_t* row_ret, int row_k, void* const* dst,
                                    uint32_t* const* counters, int nranks, uint32_t* err, cudaStream_t st,
                                    uint32_t* local_count) {
  VMC_CHECK(rows_total > 0 && N > 0 && K > 0 && groups > 0 && max_rows > 0, "gemm_rowscatter: empty problem");
  VMC_CHECK(nranks >= 1 && nranks <= 8 && row_k >= 1 && row_k <= 8, "gemm_rowscatter: bad ranks / k");
  if (bn <= 0) bn = gemm_pick_bn(max_rows);
  const int chunk = wf_chunk(wf);
  GemmArgs a = {};
  a.w = static_cast<const uint8_t*>(w_tiled);
  a.N = N;
  a.K = K;
  a.M = rows_total;
  a.KC = (K + chunk - 1) / chunk;
  a.chunks_per_split = a.KC;
  a.splits = 1;
  a.n_tiles = (N + 127) / 128;
  a.m_tiles = (max_rows + bn - 1) / bn;
  a.units = groups * a.n_tiles * a.m_tiles;
  a.out = nullptr;
  a.ldo = N;
  a.out_mode = kGemmOutRowScatterBF16;
  a.err = err;
  a.trace = g_gemm_trace;
  a.bn = bn;
  a.groups = groups;
  a.grp_count = counts;
  a.grp_offset = offsets;
  a.grp_w_stride = w_group_stride;
  for (int q = 0; q < 8; ++q) {
    a.scat[q] = q < nranks ? dst[q] : nullptr;
    a.scat_count[q] = q < nranks ? counters[q] : nullptr;
  }
  a.scat_nranks = nranks;
  a.scat_local = local_count;
  a.row_ret = row_ret;
  a.row_k = row_k;
  CUtensorMap map;
  make_act_tensor_map(&map, x, rows_total, K, ldx, bn);
  return dispatch_wf(wf, bn, map, a, st);
}

int gemm_smem_bytes(int wf, int bn) {
  return (wf != kWfBF16 && bn <= 64) ? make_dplan(wf, bn).total() : make_plan(wf, bn).total();
}

}  // namespace vmc
