// Split-KV paged decode attention behind a plain C entry point that allocates nothing.
//
// This entry point has no counterpart in the reference: the reference's decode attention
// (ggml-cuda flash_attn_ext_vec, and its split-K "fixup" buffers) always takes its scratch from
// ggml's per-call pool allocator.
//
// Why it exists. The regular entry point (paged_attention in attention.cu, reached from Python)
// expects the caller to pass the split-KV partial buffers, which the model allocates once through
// PyTorch. Some callers have no allocator they may use at the moment they need attention: a host
// runtime written in plain C that links only this library (no PyTorch, no caching allocator), a
// watchdog or error-recovery path that runs while device memory is exhausted, or code that must
// not create new allocations while another component is recording or replaying work on the
// device. For them this variant keeps its partials in a fixed, file-scope device array that is
// part of the loaded module, so a call only looks up that array's address (once per device) and
// launches the same kernels as the regular path.
//
// Contract:
//  * Capacity: the scratch holds kNoAllocScratchFloats fp32 values (4 MiB). A call needs
//    splits * total_tokens * Hq * D values for the partial outputs plus splits * total_tokens * Hq
//    log-sum-exps (rounded up to 64 values); larger requests are rejected with
//    kNoAllocErrTooLarge and a message, nothing is launched.
//  * Nothing has to start at zero: for every (split, token, head) row that the combine step reads,
//    the decode kernel of the same call writes both the partial output and its log-sum-exp (an
//    empty split writes a zero output and -inf), so stale values from an earlier call are never
//    read.
//  * One scratch per device, no locking on the device side: two calls on the same device whose
//    kernels may overlap (different streams with no ordering between them, or several host
//    threads) race on the scratch and corrupt each other's results. Serialise them, e.g. issue
//    them on one stream.
//  * Query layout: request r owns rows r * q_len .. r * q_len + q_len - 1, i.e. q_start must hold
//    exactly 0, q_len, 2 * q_len, ... (the scratch is sized from num_reqs * q_len rows). The decode
//    kernel skips partial rows past that count, so a larger q_start cannot write outside the
//    scratch, but its rows are then missing from the output.
//  * The first call on each device does the set-up: with that device current it asks the runtime
//    for the address of the scratch array (cudaGetSymbolAddress) and caches it. Make that first
//    call on a device outside any stream capture. The cached address belongs to the device's
//    primary context: do not keep using the entry point across cudaDeviceReset().
//  * Errors are returned, never thrown: 0 on success, a negative kNoAllocErr* code otherwise, with
//    a message written to the caller's buffer (errbuf, errbuf_len; may be null).
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <exception>
#include <mutex>

#include "attention.h"
#include "attention_noalloc.h"

namespace {

constexpr size_t kNoAllocScratchFloats = size_t(1) << 20;  // 4 MiB of fp32
constexpr int kNoAllocMaxDevices = 64;

enum : int {
  kNoAllocOk = VMC_NOALLOC_OK,
  kNoAllocErrArgs = VMC_NOALLOC_ERR_ARGS,
  kNoAllocErrTooLarge = VMC_NOALLOC_ERR_TOO_LARGE,
  kNoAllocErrSetup = VMC_NOALLOC_ERR_SETUP,
  kNoAllocErrLaunch = VMC_NOALLOC_ERR_LAUNCH,
};

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

float* g_scratch_ptr[kNoAllocMaxDevices] = {};
std::mutex g_setup_mu;

struct ErrSink {
  char* buf;
  int len;
  int fail(int code, const char* msg) const {
    if (buf && len > 0) std::snprintf(buf, static_cast<size_t>(len), "%s", msg);
    return code;
  }
};

// Address of this device's scratch; resolved once per device with that device current.
int scratch_for_current_device(float** out, const ErrSink& err) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return err.fail(kNoAllocErrSetup, cudaGetErrorString(e));
  if (dev < 0 || dev >= kNoAllocMaxDevices) return err.fail(kNoAllocErrSetup, "device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      char msg[160];
      std::snprintf(msg, sizeof(msg), "cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return err.fail(kNoAllocErrSetup, msg);
    }
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return kNoAllocOk;
}

}  // namespace

extern "C" {

// Decode attention for num_reqs requests with q_len tokens each (their tokens are rows
// 0 .. num_reqs * q_len - 1 of q/out), KV split into `splits` ranges per request and merged.
// Arguments mirror paged_attention (attention.h) for the decode case; all pointers are device
// pointers, `stream` is a cudaStream_t (0 = legacy default stream). On failure a message is
// written to errbuf (errbuf_len bytes, may be null).
__attribute__((visibility("default"))) int vmc_paged_decode_attention_noalloc(
    const void* q, const void* kv, const int32_t* q_start, const int32_t* ctx_len, const int32_t* block_tables,
    int max_blocks, int num_reqs, int q_len, int Hq, int Hkv, int D, float scale, int splits, void* out,
    void* stream, char* errbuf, int errbuf_len) {
  const ErrSink err{errbuf, errbuf_len};
  if (!q || !kv || !q_start || !ctx_len || !block_tables || !out) return err.fail(kNoAllocErrArgs, "null pointer argument");
  if (num_reqs <= 0 || q_len <= 0 || Hq <= 0 || Hkv <= 0 || max_blocks <= 0 || splits < 1)
    return err.fail(kNoAllocErrArgs, "num_reqs, q_len, Hq, Hkv, max_blocks must be positive and splits >= 1");
  if (D != 32 && D != 64 && D != 128) return err.fail(kNoAllocErrArgs, "head dim must be 32, 64 or 128");
  if (Hq % Hkv != 0 || q_len * (Hq / Hkv) > 16)
    return err.fail(kNoAllocErrArgs, "Hq must be a multiple of Hkv and q_len * Hq / Hkv <= 16");
  const size_t total_tokens = static_cast<size_t>(num_reqs) * static_cast<size_t>(q_len);
  const size_t rows = static_cast<size_t>(splits) * total_tokens * static_cast<size_t>(Hq);
  const size_t lse_floats = (rows + 63) / 64 * 64;  // keeps the partial outputs 256-byte aligned
  const size_t need = lse_floats + rows * static_cast<size_t>(D);
  if (need > kNoAllocScratchFloats) {
    char msg[160];
    std::snprintf(msg, sizeof(msg),
                  "split-KV scratch needs %zu floats, the fixed scratch holds %zu; lower splits or batch", need,
                  kNoAllocScratchFloats);
    return err.fail(kNoAllocErrTooLarge, msg);
  }
  float* scratch = nullptr;
  int rc = scratch_for_current_device(&scratch, err);
  if (rc != kNoAllocOk) return rc;

  vmc::AttnLaunch a;
  a.q = q;
  a.kv = kv;
  a.q_start = q_start;
  a.ctx_len = ctx_len;
  a.block_tables = block_tables;
  a.max_blocks = max_blocks;
  a.num_reqs = num_reqs;
  a.req_offset = 0;
  a.max_qlen = q_len;
  a.total_tokens = static_cast<int>(total_tokens);
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.D = D;
  a.scale = scale;
  a.decode = true;
  a.splits = splits;
  a.part_lse = scratch;
  a.part_o = scratch + lse_floats;
  a.out = out;
  try {
    vmc::paged_attention(a, static_cast<cudaStream_t>(stream));
  } catch (const std::exception& ex) {
    return err.fail(kNoAllocErrLaunch, ex.what());
  }
  return kNoAllocOk;
}

}  // extern "C"
