// C interface of the allocation-free split-KV decode attention (attention_noalloc.cu). Usable from
// plain C: no C++ types, no PyTorch.
//
// This entry point has no counterpart in the reference.
#ifndef VMC_ATTENTION_NOALLOC_H_
#define VMC_ATTENTION_NOALLOC_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// Return codes.
#define VMC_NOALLOC_OK 0
#define VMC_NOALLOC_ERR_ARGS (-1)
#define VMC_NOALLOC_ERR_TOO_LARGE (-2)
#define VMC_NOALLOC_ERR_SETUP (-3)
#define VMC_NOALLOC_ERR_LAUNCH (-4)

// Decode attention of num_reqs requests with exactly q_len query tokens each: request r's tokens are
// rows r * q_len .. r * q_len + q_len - 1 of q and out, so q_start (device, num_reqs + 1 entries) must
// hold exactly 0, q_len, 2 * q_len, ...; rows of a request with fewer tokens would be combined from
// stale scratch. Every pointer is a device pointer; `stream` is a cudaStream_t (null = legacy default
// stream). Returns VMC_NOALLOC_OK or a negative code with a message in errbuf (may be null).
int vmc_paged_decode_attention_noalloc(const void* q, const void* kv, const int32_t* q_start,
                                       const int32_t* ctx_len, const int32_t* block_tables, int max_blocks,
                                       int num_reqs, int q_len, int Hq, int Hkv, int D, float scale, int splits,
                                       void* out, void* stream, char* errbuf, int errbuf_len);

#ifdef __cplusplus
}
#endif

#endif  // VMC_ATTENTION_NOALLOC_H_
