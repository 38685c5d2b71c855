// Link-time stand-ins for the two vm_c TurboQuant-bridge hooks that the reference's patched libllama
// references (include/vm_c/official/vm_c_llama_graph_ext.h). Their real definitions live in
// src/official/turboquant_kv_bridge.cpp, which needs the whole vm_c engine. libllama calls them only
// when a context is created with a TurboQuant bridge (cparams.vm_c_tq_bridge != nullptr,
// llama-graph.cpp:2288-2290); the reference arm runs the bf16 KV cache, so they are never called.
#include <cstdint>

struct ggml_tensor;

extern "C" ggml_tensor* vm_c_tq_bridge_kv_tensor(void*, int32_t) { return nullptr; }
extern "C" bool vm_c_tq_bridge_layer_uses_turboquant(void*, int32_t) { return false; }
