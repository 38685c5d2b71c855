// Fused-dequant GEMM on the 5th-generation tensor cores: out[M, N] = X[M, K] @ W[N, K]^T.
//
// B200-native replacement for the reference's quantized matmul path (ggml-cuda mul_mat_q /
// mul_mat_vec_q, ggml-cuda/mmq.cuh:3542, mmvq.cu:398, and cuBLAS for F16/BF16 weights), which on
// sm_100 runs as Ampere-class mma.sync / dp4a code.
//
// Design ("swap-AB"): the weight tile is the UMMA A operand (M_mma = 128 output features), the
// activation tile is the B operand (N_mma = BN tokens, 16..256), the fp32 accumulator lives in TMEM.
// Warp roles in a 320-thread CTA:
//   warp 0      producer: TMA 2-D loads of activation tiles (128B swizzle, zero fill past M/K) and
//               one cp.async.bulk per weight tile (tiles are stored contiguously, see
//               weight_formats.cuh); bf16 weights go straight into the A stage.
//   warp 1      allocates TMEM; one elected lane issues tcgen05.mma (K=16 per instruction) and
//               tcgen05.commit to release stages.
//   warps 2-9   dequantize GGUF blocks from the raw stage into the swizzled bf16 A stage
//               (packed bf16x2 integer tricks, see the per-format functions), then run the
//               epilogue: tcgen05.ld -> bf16 store, fp32 red.add (split-K), or fused SwiGLU.
// Every wait is bounded; on expiry the CTA records an error code and unwinds (TMEM is freed).
#include <cuda.h>

#include "common.cuh"
#include "gemm_tcgen05.h"
#include "weight_formats.cuh"

namespace vmc {
namespace {

constexpr int kThreads = 320;
constexpr int kDequantWarps = 8;
constexpr int kFirstDqWarp = 2;

struct GemmSmemPlan {
  int stages;      // A/B pipeline stages (64-K each)
  int raw_stages;  // raw quant tile stages (256-K each)
  int bn;
  int wf;
  __host__ __device__ int a_bytes() const { return 128 * 128; }
  __host__ __device__ int b_bytes() const { return bn * 128; }
  __host__ __device__ int raw_bytes() const { return wf == kWfBF16 ? 0 : wf_tile_bytes(wf); }
  __host__ __device__ int off_b() const { return stages * a_bytes(); }
  __host__ __device__ int off_raw() const { return off_b() + stages * b_bytes(); }
  __host__ __device__ int off_bar() const { return off_raw() + raw_stages * raw_bytes(); }
  __host__ __device__ int total() const { return off_bar() + (2 * stages + 2 * raw_stages + 2) * 8 + 16 + 1024; }
};

__host__ __device__ inline GemmSmemPlan make_plan(int wf, int bn) {
  GemmSmemPlan p;
  p.bn = bn;
  p.wf = wf;
  const int budget = 220 * 1024;
  p.raw_stages = wf == kWfBF16 ? 0 : 2;
  p.stages = 2;
  // Grow the A/B ring first, then the raw ring, while the plan fits.
  while (true) {
    GemmSmemPlan q = p;
    q.stages += 1;
    if (q.stages > 8 || q.total() > budget) break;
    p = q;
  }
  if (wf != kWfBF16) {
    while (true) {
      GemmSmemPlan q = p;
      q.raw_stages += 1;
      if (q.raw_stages > 4 || q.total() > budget) break;
      p = q;
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
__device__ __forceinline__ uint32_t bf2_mul(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hmul2(*reinterpret_cast<__nv_bfloat162*>(&a), *reinterpret_cast<__nv_bfloat162*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t bf2_splat(float f) { return pack_bf16x2(f, f); }

constexpr uint32_t kMagic128x2 = 0x43004300u;  // bf16 (128, 128); 128 + q is exact for q < 128

__device__ __forceinline__ void dq_q4k(const uint8_t* row, int s, int h, uint32_t (&o)[16]) {
  const uint32_t dd = *reinterpret_cast<const uint32_t*>(row);
  const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(dd & 0xffffu)));
  const float dmin = __half2float(__ushort_as_half(static_cast<unsigned short>(dd >> 16)));
  const uint8_t* sc = row + 4;
  const int j = 2 * s + h;
  int scv, mv;
  if (j < 4) {
    scv = sc[j] & 63;
    mv = sc[j + 4] & 63;
  } else {
    scv = (sc[j + 4] & 0x0f) | ((sc[j - 4] >> 6) << 4);
    mv = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
  }
  const uint32_t ds2 = bf2_splat(d * static_cast<float>(scv));
  const uint32_t ndm2 = bf2_splat(-dmin * static_cast<float>(mv));
  const uint4* q = reinterpret_cast<const uint4*>(row + 16 + 32 * s);
  const uint4 w0 = q[0], w1 = q[1];
  const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
  const int sh0 = h ? 4 : 0, sh1 = h ? 12 : 8;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    uint32_t p01 = ((w[i] >> sh0) & 0x000f000fu) | kMagic128x2;
    uint32_t p23 = ((w[i] >> sh1) & 0x000f000fu) | kMagic128x2;
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
      o[4 * i + p] = bf2_mul(bf2_sub(x, kOff), scale);
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
    o[2 * i] = bf2_mul(bf2_sub(y01, z01), d2);
    o[2 * i + 1] = bf2_mul(bf2_sub(y23, z23), d2);
  }
}

// ---------------------------------------------------------------------------------------------

struct GemmArgs {
  const uint8_t* w;       // tiled weights
  int N, K, M;
  int KC;                 // number of K chunks in the tiled weight (ceil(K / chunk))
  int chunks_per_split;
  void* out;
  int ldo;                // output row stride in elements
  int out_mode;           // GemmOut
  uint32_t* err;
};

template <int WF, int BN>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ CUtensorMap xmap, GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const GemmSmemPlan P = make_plan(WF, BN);
  uint8_t* sA = smem;
  uint8_t* sB = smem + P.off_b();
  uint8_t* sRaw = smem + P.off_raw();
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P.off_bar());
  uint64_t* ab_full = bars;
  uint64_t* ab_empty = bars + P.stages;
  uint64_t* raw_full = bars + 2 * P.stages;
  uint64_t* raw_empty = raw_full + P.raw_stages;
  uint64_t* acc_full = raw_empty + P.raw_stages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 2);
  volatile uint32_t* abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nt = blockIdx.x, mt = blockIdx.y;
  const int c_begin = blockIdx.z * args.chunks_per_split;
  const int c_end = min(args.KC, c_begin + args.chunks_per_split);
  const int nchunks = c_end - c_begin;
  constexpr int SUBS = (WF == kWfBF16) ? 1 : 4;  // 64-K substeps per chunk
  constexpr uint32_t kTmemCols = BN < 32 ? 32 : BN;
  const bool quant = WF != kWfBF16;

  if (threadIdx.x == 0) {
    for (int i = 0; i < P.stages; ++i) {
      mbar_init(&ab_full[i], 1 + (quant ? kDequantWarps : 0));
      mbar_init(&ab_empty[i], 1);
    }
    for (int i = 0; i < P.raw_stages; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], kDequantWarps);
    }
    mbar_init(acc_full, 1);
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

  if (nchunks > 0) {
    if (warp == 0) {
      if (lane == 0) {
        const uint64_t pol = l2_policy_evict_first();
        int stage = 0;
        uint32_t phase = 0;
        int rstage = 0;
        uint32_t rphase = 0;
        for (int c = 0; c < nchunks && !*abort_flag; ++c) {
          const int kc = c_begin + c;
          const uint8_t* wt = args.w + (static_cast<size_t>(nt) * args.KC + kc) * wf_tile_bytes(WF);
          if (quant) {
            if (!mbar_wait(&raw_empty[rstage], rphase ^ 1, args.err, kErrGemmWait)) { *abort_flag = 1; break; }
            mbar_arrive_expect_tx(&raw_full[rstage], wf_tile_bytes(WF));
            bulk_load_evict_first(sRaw + rstage * P.raw_bytes(), wt, wf_tile_bytes(WF), &raw_full[rstage], pol);
            if (++rstage == P.raw_stages) { rstage = 0; rphase ^= 1; }
          }
          for (int sub = 0; sub < SUBS; ++sub) {
            if (!mbar_wait(&ab_empty[stage], phase ^ 1, args.err, kErrGemmWait)) { *abort_flag = 1; break; }
            const uint32_t bytes = P.b_bytes() + (quant ? 0 : P.a_bytes());
            mbar_arrive_expect_tx(&ab_full[stage], bytes);
            tma_load_2d(sB + stage * P.b_bytes(), &xmap, &ab_full[stage], (kc * SUBS + sub) * 64, mt * BN);
            if (!quant) bulk_load_evict_first(sA + stage * P.a_bytes(), wt, P.a_bytes(), &ab_full[stage], pol);
            if (++stage == P.stages) { stage = 0; phase ^= 1; }
          }
        }
      }
    } else if (warp == 1) {
      if (lane == 0) {
        const uint32_t idesc = umma_idesc_bf16(128, BN);
        int stage = 0;
        uint32_t phase = 0;
        const int total = nchunks * SUBS;
        bool ok = true;
        for (int i = 0; i < total; ++i) {
          if (!mbar_wait(&ab_full[stage], phase, args.err, kErrGemmWait)) { *abort_flag = 1; ok = false; break; }
          tc_fence_after();
          const uint64_t a0 = umma_sdesc_sw128(smem_u32(sA + stage * P.a_bytes()));
          const uint64_t b0 = umma_sdesc_sw128(smem_u32(sB + stage * P.b_bytes()));
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            umma_bf16(tmem, a0 + 2 * k, b0 + 2 * k, idesc, (i > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&ab_empty[stage]);
          if (++stage == P.stages) { stage = 0; phase ^= 1; }
        }
        (void)ok;
        umma_commit(acc_full);
      }
    } else {
      // Dequant warps (quantized formats only).
      const int t = threadIdx.x - kFirstDqWarp * 32;  // 0..255
      const int r = t >> 1, h = t & 1;
      if (quant) {
        int stage = 0;
        uint32_t phase = 0;
        int rstage = 0;
        uint32_t rphase = 0;
        for (int c = 0; c < nchunks; ++c) {
          if (!mbar_wait(&raw_full[rstage], rphase, args.err, kErrGemmWait)) { *abort_flag = 1; break; }
          const uint8_t* row = sRaw + rstage * P.raw_bytes() + r * wf_row_bytes(WF);
          bool ok = true;
          for (int sub = 0; sub < SUBS; ++sub) {
            if (!mbar_wait(&ab_empty[stage], phase ^ 1, args.err, kErrGemmWait)) { *abort_flag = 1; ok = false; break; }
            uint32_t o[16];
            if (WF == kWfQ4K) dq_q4k(row, sub, h, o);
            else if (WF == kWfQ6K) dq_q6k(row, sub, h, o);
            else dq_q8_0(row, sub, h, o);
            uint8_t* a = sA + stage * P.a_bytes();
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
              *reinterpret_cast<uint4*>(a + sw128_offset(r, 4 * h + cc)) =
                  make_uint4(o[4 * cc], o[4 * cc + 1], o[4 * cc + 2], o[4 * cc + 3]);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ab_full[stage]);
            if (++stage == P.stages) { stage = 0; phase ^= 1; }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&raw_empty[rstage]);
          if (++rstage == P.raw_stages) { rstage = 0; rphase ^= 1; }
          if (!ok) break;
        }
      }
      // Epilogue: warps 2..9 -> TMEM lane quarter (warp % 4), column half ((warp - 2) / 4).
      if (mbar_wait(acc_full, 0, args.err, kErrGemmWait)) {
        tc_fence_after();
        const int q = warp & 3;
        const int half = (warp - kFirstDqWarp) >> 2;
        const int n_local = 32 * q + lane;
        constexpr int HALVES = BN >= 32 ? 2 : 1;
        constexpr int COLS = BN / HALVES;
        const int col0 = half * COLS;
        for (int cb = 0; cb < COLS && half < HALVES; cb += 16) {
          uint32_t v[16];
          tmem_ld16(tmem + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(col0 + cb), v);
          tmem_ld_wait();
          const int m_base = mt * BN + col0 + cb;
          if (args.out_mode == kGemmOutSwiGLU) {
            // Rows interleave gate (even) and up (odd) features of the same output column.
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float mine = __uint_as_float(v[j]);
              const float other = __shfl_xor_sync(0xffffffffu, mine, 1);
              const int m = m_base + j;
              if ((lane & 1) == 0 && m < args.M) {
                const float g = mine, u = other;
                const float y = g / (1.f + __expf(-g)) * u;
                const int f = nt * 64 + (n_local >> 1);
                if (f < args.N / 2)
                  reinterpret_cast<__nv_bfloat16*>(args.out)[static_cast<size_t>(m) * args.ldo + f] = __float2bfloat16(y);
              }
            }
          } else {
            const int n = nt * 128 + n_local;
            if (n < args.N) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int m = m_base + j;
                if (m < args.M) {
                  const float y = __uint_as_float(v[j]);
                  const size_t idx = static_cast<size_t>(m) * args.ldo + n;
                  if (args.out_mode == kGemmOutF32Add) atomicAdd(reinterpret_cast<float*>(args.out) + idx, y);
                  else if (args.out_mode == kGemmOutF32) reinterpret_cast<float*>(args.out)[idx] = y;
                  else reinterpret_cast<__nv_bfloat16*>(args.out)[idx] = __float2bfloat16(y);
                }
              }
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
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

template <int WF, int BN>
void launch(const CUtensorMap& map, const GemmArgs& a, int splits, cudaStream_t st) {
  const GemmSmemPlan P = make_plan(WF, BN);
  static bool configured = false;
  if (!configured) {
    VMC_CUDA_CHECK(cudaFuncSetAttribute(gemm_kernel<WF, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, P.total()));
    configured = true;
  }
  dim3 grid((a.N + 127) / 128, (a.M + BN - 1) / BN, splits);
  gemm_kernel<WF, BN><<<grid, kThreads, P.total(), st>>>(map, a);
  VMC_CUDA_CHECK(cudaGetLastError());
}

template <int WF>
void dispatch_bn(int bn, const CUtensorMap& map, const GemmArgs& a, int splits, cudaStream_t st) {
  switch (bn) {
    case 16: launch<WF, 16>(map, a, splits, st); break;
    case 32: launch<WF, 32>(map, a, splits, st); break;
    case 64: launch<WF, 64>(map, a, splits, st); break;
    case 128: launch<WF, 128>(map, a, splits, st); break;
    case 256: launch<WF, 256>(map, a, splits, st); break;
    default: throw std::runtime_error("gemm: unsupported BN");
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

int gemm_pick_bn(int M) {
  if (M <= 16) return 16;
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  if (M <= 128) return 128;
  return 256;
}

void gemm_tcgen05(int wf, const void* w_tiled, int N, int K, const void* x, int M, int ldx, void* out, int ldo,
                  int out_mode, int splits, int bn, uint32_t* err, cudaStream_t st) {
  VMC_CHECK(M > 0 && N > 0 && K > 0, "gemm: empty problem");
  if (bn <= 0) bn = gemm_pick_bn(M);
  const int chunk = wf_chunk(wf);
  const int KC = (K + chunk - 1) / chunk;
  if (splits < 1) splits = 1;
  if (splits > KC) splits = KC;
  VMC_CHECK(splits == 1 || out_mode == kGemmOutF32Add, "gemm: split-K needs the fp32 accumulate output mode");
  GemmArgs a;
  a.w = static_cast<const uint8_t*>(w_tiled);
  a.N = N;
  a.K = K;
  a.M = M;
  a.KC = KC;
  a.chunks_per_split = (KC + splits - 1) / splits;
  splits = (KC + a.chunks_per_split - 1) / a.chunks_per_split;
  a.out = out;
  a.ldo = ldo;
  a.out_mode = out_mode;
  a.err = err;
  CUtensorMap map;
  make_act_tensor_map(&map, x, M, K, ldx, bn);
  switch (wf) {
    case kWfBF16: dispatch_bn<kWfBF16>(bn, map, a, splits, st); break;
    case kWfQ4K: dispatch_bn<kWfQ4K>(bn, map, a, splits, st); break;
    case kWfQ6K: dispatch_bn<kWfQ6K>(bn, map, a, splits, st); break;
    case kWfQ8_0: dispatch_bn<kWfQ8_0>(bn, map, a, splits, st); break;
    default: throw std::runtime_error("gemm: unknown weight format");
  }
}

int gemm_smem_bytes(int wf, int bn) { return make_plan(wf, bn).total(); }

}  // namespace vmc
