// Python bindings of the native host runtime (GGUF container, quant codecs, paged block manager,
// scheduler and batch-metadata builder). Host-only C++; imports without CUDA.
#include <pybind11/functional.h>
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstring>
#include <thread>

#include "block_manager.hpp"
#include "gguf.hpp"
#include "quants.hpp"
#include "safetensors.hpp"
#include "scheduler.hpp"
#include "tokenizer.hpp"
#include "turboquant.hpp"

namespace py = pybind11;
using namespace vmc;

namespace {

py::object value_to_py(const GValue& v) {
  switch (v.type) {
    case GValueType::UINT8: case GValueType::UINT16: case GValueType::UINT32: case GValueType::UINT64:
      return py::int_(v.u);
    case GValueType::INT8: case GValueType::INT16: case GValueType::INT32: case GValueType::INT64:
      return py::int_(v.i);
    case GValueType::FLOAT32: case GValueType::FLOAT64: return py::float_(v.f);
    case GValueType::BOOL: return py::bool_(v.b);
    case GValueType::STRING: return py::bytes(v.s);
    case GValueType::ARRAY: {
      py::list out;
      switch (v.elem_type) {
        case GValueType::STRING: for (auto& s : v.as) out.append(py::bytes(s)); break;
        case GValueType::BOOL: for (auto b : v.ab) out.append(py::bool_(b != 0)); break;
        case GValueType::FLOAT32: case GValueType::FLOAT64: for (auto f : v.af) out.append(py::float_(f)); break;
        case GValueType::UINT8: case GValueType::UINT16: case GValueType::UINT32: case GValueType::UINT64:
          for (auto u : v.au) out.append(py::int_(u));
          break;
        default: for (auto i : v.ai) out.append(py::int_(i)); break;
      }
      return out;
    }
    default: return py::none();
  }
}

GValue py_to_value(uint32_t type, py::handle obj, uint32_t elem_type) {
  GValue v;
  v.type = static_cast<GValueType>(type);
  auto scalar = [](GValue& dst, GValueType t, py::handle o, bool arr) {
    switch (t) {
      case GValueType::UINT8: case GValueType::UINT16: case GValueType::UINT32: case GValueType::UINT64:
        if (arr) dst.au.push_back(o.cast<uint64_t>()); else dst.u = o.cast<uint64_t>();
        break;
      case GValueType::INT8: case GValueType::INT16: case GValueType::INT32: case GValueType::INT64:
        if (arr) dst.ai.push_back(o.cast<int64_t>()); else dst.i = o.cast<int64_t>();
        break;
      case GValueType::FLOAT32: case GValueType::FLOAT64:
        if (arr) dst.af.push_back(o.cast<double>()); else dst.f = o.cast<double>();
        break;
      case GValueType::BOOL:
        if (arr) dst.ab.push_back(o.cast<bool>() ? 1 : 0); else dst.b = o.cast<bool>();
        break;
      case GValueType::STRING: {
        std::string s = py::isinstance<py::bytes>(o) ? o.cast<std::string>() : py::str(o).cast<std::string>();
        if (arr) dst.as.push_back(std::move(s)); else dst.s = std::move(s);
        break;
      }
      default: throw std::runtime_error("unsupported GGUF value type");
    }
  };
  if (v.type == GValueType::ARRAY) {
    v.elem_type = static_cast<GValueType>(elem_type);
    for (auto item : obj) scalar(v, v.elem_type, item, true);
  } else {
    scalar(v, v.type, obj, false);
  }
  return v;
}

int default_threads() {
  unsigned n = std::thread::hardware_concurrency();
  return n == 0 ? 4 : static_cast<int>(std::min(n, 64u));
}

}  // namespace

PYBIND11_MODULE(_host, m) {
  m.doc() = "vm_c_b200 native host runtime";

  // ---------------- GGUF ----------------
  py::class_<GgufFile, std::shared_ptr<GgufFile>>(m, "GgufFile")
      .def_static("open", &GgufFile::open, py::arg("path"))
      .def_property_readonly("version", &GgufFile::version)
      .def_property_readonly("alignment", &GgufFile::alignment)
      .def_property_readonly("data_offset", &GgufFile::data_offset)
      .def_property_readonly("path", &GgufFile::path)
      .def("keys", &GgufFile::keys)
      .def("has", &GgufFile::has)
      .def("get", [](const GgufFile& f, const std::string& k) { return value_to_py(f.get(k)); })
      .def("value_type", [](const GgufFile& f, const std::string& k) {
        const auto& v = f.get(k);
        return py::make_tuple(static_cast<uint32_t>(v.type), static_cast<uint32_t>(v.elem_type));
      })
      .def("tensors", [](const GgufFile& f) {
        py::list out;
        for (auto& t : f.tensors()) {
          py::dict d;
          d["name"] = t.name;
          d["ne"] = t.ne;
          d["type"] = static_cast<uint32_t>(t.type);
          d["offset"] = t.offset;
          d["nbytes"] = t.nbytes;
          out.append(d);
        }
        return out;
      })
      // Zero-copy read-only view of a tensor's bytes (keeps the mapping alive).
      .def("tensor_bytes", [](std::shared_ptr<GgufFile> f, const std::string& name) {
        const GTensorInfo* t = f->find_tensor(name);
        if (!t) throw py::key_error("no tensor " + name);
        auto holder = py::cast(f);
        py::array_t<uint8_t> arr({static_cast<py::ssize_t>(t->nbytes)}, {1}, f->tensor_data(*t), holder);
        py::detail::array_proxy(arr.ptr())->flags &= ~py::detail::npy_api::NPY_ARRAY_WRITEABLE_;
        return arr;
      });

  // ---------------- safetensors ----------------
  py::class_<SafetensorsFile, std::shared_ptr<SafetensorsFile>>(m, "SafetensorsFile")
      .def_static("open", &SafetensorsFile::open, py::arg("path"))
      .def_property_readonly("path", &SafetensorsFile::path)
      .def("metadata", &SafetensorsFile::metadata)
      .def("tensors", [](const SafetensorsFile& f) {
        py::list out;
        for (auto& t : f.tensors()) {
          py::dict d;
          d["name"] = t.name;
          d["dtype"] = t.dtype;
          d["shape"] = t.shape;
          d["begin"] = t.begin;
          d["end"] = t.end;
          out.append(d);
        }
        return out;
      })
      // Zero-copy read-only view of a tensor's bytes (keeps the mapping alive).
      .def("tensor_bytes", [](std::shared_ptr<SafetensorsFile> f, const std::string& name) {
        const StTensorInfo* t = f->find(name);
        if (!t) throw py::key_error("no tensor " + name);
        auto holder = py::cast(f);
        py::array_t<uint8_t> arr({static_cast<py::ssize_t>(t->end - t->begin)}, {1}, f->data(*t), holder);
        py::detail::array_proxy(arr.ptr())->flags &= ~py::detail::npy_api::NPY_ARRAY_WRITEABLE_;
        return arr;
      });

  py::class_<GgufWriter>(m, "GgufWriter")
      .def(py::init<uint64_t>(), py::arg("alignment") = 32)
      .def("set", [](GgufWriter& w, const std::string& key, uint32_t type, py::handle value, uint32_t elem_type) {
        w.set(key, py_to_value(type, value, elem_type));
      }, py::arg("key"), py::arg("type"), py::arg("value"), py::arg("elem_type") = 0)
      .def("add_tensor", [](GgufWriter& w, const std::string& name, std::vector<int64_t> ne, uint32_t type) {
        w.add_tensor(name, ne, static_cast<GType>(type));
      })
      // producer(index) -> a buffer (bytes / numpy array) with exactly the tensor's byte count.
      .def("write", [](GgufWriter& w, const std::string& path, py::function producer) {
        w.write(path, [&](size_t i, uint8_t* dst, uint64_t nbytes) {
          py::object obj = producer(i);
          py::buffer_info bi = py::buffer(obj).request();
          uint64_t have = static_cast<uint64_t>(bi.size) * static_cast<uint64_t>(bi.itemsize);
          if (have != nbytes) throw std::runtime_error("GgufWriter: tensor " + std::to_string(i) + " has " + std::to_string(have) + " bytes, expected " + std::to_string(nbytes));
          std::memcpy(dst, bi.ptr, nbytes);
        });
      });

  m.def("type_traits", [](uint32_t t) {
    auto tr = gtype_traits(static_cast<GType>(t));
    return py::make_tuple(std::string(tr.name), tr.block_elems, tr.block_bytes);
  });
  m.def("row_bytes", [](uint32_t t, int64_t n) { return gtype_row_bytes(static_cast<GType>(t), n); });

  // ---------------- quant codecs ----------------
  m.def("tq_layout", [](const std::string& method, int head_dim) {
    const vmc::TqLayout l = vmc::TqLayout::from_method(head_dim, method);
    py::dict d;
    d["head_dim"] = l.head_dim;
    d["key_bits"] = l.key_bits;
    d["value_bits"] = l.value_bits;
    d["norm_correction"] = l.norm_correction;
    d["key_fp8"] = l.key_fp8;
    d["n_centroids"] = l.n_centroids;
    d["mse_bytes"] = l.mse_bytes;
    d["key_packed"] = l.key_packed;
    d["val_bytes"] = l.val_bytes;
    d["value_packed"] = l.value_packed;
    d["slot"] = l.slot;
    d["slot_aligned"] = l.slot_aligned;
    return d;
  });
  m.def("is_turboquant_method", &vmc::is_turboquant_method);
  m.def("lloyd_max_gaussian", &vmc::lloyd_max_gaussian, py::arg("bits"), py::arg("sigma"));
  m.def("dequantize", [](uint32_t type, py::buffer src, int64_t rows, int64_t row_elems, int threads) {
    py::buffer_info bi = src.request();
    size_t need = gtype_row_bytes(static_cast<GType>(type), row_elems) * static_cast<size_t>(rows);
    if (static_cast<size_t>(bi.size * bi.itemsize) < need) throw std::runtime_error("dequantize: source too small");
    py::array_t<float> out({rows, row_elems});
    {
      py::gil_scoped_release nogil;
      dequantize_tensor(static_cast<GType>(type), bi.ptr, out.mutable_data(), rows, row_elems, threads > 0 ? threads : default_threads());
    }
    return out;
  }, py::arg("type"), py::arg("src"), py::arg("rows"), py::arg("row_elems"), py::arg("threads") = 0);

  m.def("quantize", [](uint32_t type, py::array_t<float, py::array::c_style | py::array::forcecast> src, int threads) {
    if (src.ndim() != 2) throw std::runtime_error("quantize: expected a 2-D float32 array");
    int64_t rows = src.shape(0), row_elems = src.shape(1);
    size_t rb = gtype_row_bytes(static_cast<GType>(type), row_elems);
    py::array_t<uint8_t> out({static_cast<py::ssize_t>(rows), static_cast<py::ssize_t>(rb)});
    {
      py::gil_scoped_release nogil;
      quantize_tensor(static_cast<GType>(type), src.data(), out.mutable_data(), rows, row_elems, threads > 0 ? threads : default_threads());
    }
    return out;
  }, py::arg("type"), py::arg("src"), py::arg("threads") = 0);
  m.def("can_quantize", [](uint32_t t) { return can_quantize(static_cast<GType>(t)); });

  // ---------------- tokenizer core ----------------
  py::class_<BpeTokenizer>(m, "BpeTokenizer")
      .def(py::init([](const std::vector<py::bytes>& toks, const std::vector<float>& scores,
                       const std::vector<py::bytes>& merges, const std::string& model) {
        std::vector<std::string> t, mg;
        t.reserve(toks.size());
        for (auto& x : toks) t.push_back(x);
        for (auto& x : merges) mg.push_back(x);
        return new BpeTokenizer(t, scores, mg, model);
      }))
      .def("encode_piece", [](const BpeTokenizer& b, py::bytes text) { return b.encode_piece(text); })
      .def("token_id", [](const BpeTokenizer& b, py::bytes piece) { return b.token_id(piece); })
      .def("set_unk", &BpeTokenizer::set_unk)
      .def_property_readonly("vocab_size", &BpeTokenizer::vocab_size);

  // ---------------- block manager ----------------
  py::class_<BlockManager, std::shared_ptr<BlockManager>>(m, "BlockManager")
      .def(py::init<int64_t, int, bool>(), py::arg("num_blocks"), py::arg("block_size"), py::arg("enable_prefix_caching") = true)
      .def_property_readonly("block_size", &BlockManager::block_size)
      .def_property_readonly("num_blocks", &BlockManager::num_blocks)
      .def_property_readonly("num_free_blocks", &BlockManager::num_free_blocks)
      .def_property_readonly("num_cached_blocks", &BlockManager::num_cached_blocks)
      .def("usage", &BlockManager::usage)
      .def("allocate", &BlockManager::allocate, py::arg("rid"), py::arg("num_tokens"), py::arg("hit_blocks") = std::vector<int32_t>{})
      .def("can_allocate", &BlockManager::can_allocate)
      .def("free", &BlockManager::free)
      .def("trim", &BlockManager::trim)
      .def("blocks_of", &BlockManager::blocks_of)
      .def("find_longest_prefix_hit", [](const BlockManager& b, const std::vector<uint64_t>& h, int max_blocks) {
        std::vector<int32_t> out;
        b.find_longest_prefix_hit(h, max_blocks, out);
        return out;
      })
      .def("cache_full_blocks", &BlockManager::cache_full_blocks)
      .def("reset_prefix_cache", &BlockManager::reset_prefix_cache)
      .def_static("block_hashes", [](const std::vector<int32_t>& toks, int bs) {
        return BlockManager::block_hashes(toks.data(), static_cast<int64_t>(toks.size()), bs);
      });

  // ---------------- scheduler ----------------
  py::class_<SchedulerConfig>(m, "SchedulerConfig")
      .def(py::init<>())
      .def_readwrite("max_num_seqs", &SchedulerConfig::max_num_seqs)
      .def_readwrite("max_num_batched_tokens", &SchedulerConfig::max_num_batched_tokens)
      .def_readwrite("max_model_len", &SchedulerConfig::max_model_len)
      .def_readwrite("enable_chunked_prefill", &SchedulerConfig::enable_chunked_prefill)
      .def_readwrite("long_prefill_token_threshold", &SchedulerConfig::long_prefill_token_threshold)
      .def_readwrite("decode_first", &SchedulerConfig::decode_first)
      .def_readwrite("max_prefill_per_batch", &SchedulerConfig::max_prefill_per_batch)
      .def_readwrite("decode_latency_target_ms", &SchedulerConfig::decode_latency_target_ms)
      .def_readwrite("preempt_prefill_on_latency", &SchedulerConfig::preempt_prefill_on_latency)
      .def_readwrite("decode_reserved_tokens", &SchedulerConfig::decode_reserved_tokens)
      .def_readwrite("num_lookahead_tokens", &SchedulerConfig::num_lookahead_tokens);

  py::class_<SeqParams>(m, "SeqParams")
      .def(py::init<>())
      .def_readwrite("max_tokens", &SeqParams::max_tokens)
      .def_readwrite("min_tokens", &SeqParams::min_tokens)
      .def_readwrite("ignore_eos", &SeqParams::ignore_eos)
      .def_readwrite("stop_token_ids", &SeqParams::stop_token_ids)
      .def_readwrite("eos_token_ids", &SeqParams::eos_token_ids);

  py::class_<PlanEntry>(m, "PlanEntry")
      .def_readonly("id", &PlanEntry::id)
      .def_readonly("slot", &PlanEntry::slot)
      .def_readonly("num_tokens", &PlanEntry::num_tokens)
      .def_readonly("start", &PlanEntry::start)
      .def_readonly("sample", &PlanEntry::sample)
      .def_readonly("is_decode", &PlanEntry::is_decode);

  py::class_<Plan>(m, "Plan")
      .def_readonly("entries", &Plan::entries)
      .def_readonly("total_tokens", &Plan::total_tokens)
      .def_readonly("num_decode", &Plan::num_decode)
      .def_readonly("num_sample", &Plan::num_sample)
      .def_readonly("num_cached_tokens", &Plan::num_cached_tokens)
      .def_readonly("preempted", &Plan::preempted)
      .def_readonly("decode_latency_preempt", &Plan::decode_latency_preempt)
      .def("sample_ids", [](const Plan& p) {
        std::vector<int64_t> ids;
        for (auto& e : p.entries) if (e.sample) ids.push_back(e.id);
        return ids;
      })
      .def("sample_slots", [](const Plan& p) {
        std::vector<int32_t> s;
        for (auto& e : p.entries) if (e.sample) s.push_back(e.slot);
        return s;
      })
      .def("__len__", [](const Plan& p) { return p.entries.size(); });

  py::class_<BatchLayout>(m, "BatchLayout")
      .def(py::init([](int mt, int mr, int mb) { return BatchLayout{mt, mr, mb}; }), py::arg("max_tokens"), py::arg("max_reqs"), py::arg("max_blocks_per_seq"))
      .def_readonly("max_tokens", &BatchLayout::max_tokens)
      .def_readonly("max_reqs", &BatchLayout::max_reqs)
      .def_readonly("max_blocks_per_seq", &BatchLayout::max_blocks_per_seq)
      .def_property_readonly("off_input_ids", &BatchLayout::off_input_ids)
      .def_property_readonly("off_positions", &BatchLayout::off_positions)
      .def_property_readonly("off_slot_mapping", &BatchLayout::off_slot_mapping)
      .def_property_readonly("off_q_start", &BatchLayout::off_q_start)
      .def_property_readonly("off_ctx_len", &BatchLayout::off_ctx_len)
      .def_property_readonly("off_seq_slot", &BatchLayout::off_seq_slot)
      .def_property_readonly("off_logits_idx", &BatchLayout::off_logits_idx)
      .def_property_readonly("off_sample_req", &BatchLayout::off_sample_req)
      .def_property_readonly("off_counts", &BatchLayout::off_counts)
      .def_property_readonly("off_block_tables", &BatchLayout::off_block_tables)
      .def_property_readonly("total", &BatchLayout::total);

  py::class_<Scheduler>(m, "Scheduler")
      .def(py::init<const SchedulerConfig&, std::shared_ptr<BlockManager>>())
      .def("add_request", &Scheduler::add_request)
      .def("abort_request", &Scheduler::abort_request)
      .def("schedule", &Scheduler::schedule)
      // buf_addr: address of a host buffer with layout.total int32 elements (e.g. a pinned tensor).
      .def("build_batch", [](const Scheduler& s, const Plan& p, const BatchLayout& L, uintptr_t buf_addr, int pad) {
        s.build_batch(p, L, reinterpret_cast<int32_t*>(buf_addr), pad);
      }, py::arg("plan"), py::arg("layout"), py::arg("buf_addr"), py::arg("pad_to_reqs") = 0)
      // flat: new tokens of all sampled entries concatenated; per_entry: count per sampled entry
      // (default one each).
      .def("update", [](Scheduler& s, const Plan& p, py::array_t<int32_t, py::array::c_style | py::array::forcecast> flat,
                        py::object per_entry) {
        std::vector<std::vector<int32_t>> toks;
        const int32_t* f = flat.data();
        py::ssize_t n = flat.size();
        if (per_entry.is_none()) {
          toks.reserve(static_cast<size_t>(n));
          for (py::ssize_t i = 0; i < n; ++i) toks.push_back({f[i]});
        } else {
          auto counts = per_entry.cast<std::vector<int>>();
          py::ssize_t o = 0;
          for (int c : counts) {
            if (o + c > n) throw std::runtime_error("update: per-entry counts exceed the token array");
            toks.emplace_back(f + o, f + o + c);
            o += c;
          }
        }
        auto ev = s.update(p, toks);
        py::list out;
        for (auto& e : ev) out.append(py::make_tuple(e.id, e.tokens, e.finished, static_cast<int>(e.reason)));
        return out;
      }, py::arg("plan"), py::arg("tokens"), py::arg("per_entry") = py::none())
      .def("finish_request", [](Scheduler& s, int64_t id, int reason) { s.finish_request(id, static_cast<FinishReason>(reason)); })
      .def("release", &Scheduler::release)
      .def_property_readonly("num_waiting", &Scheduler::num_waiting)
      .def_property_readonly("num_running", &Scheduler::num_running)
      .def("has_unfinished", &Scheduler::has_unfinished)
      .def("seq_info", [](const Scheduler& s, int64_t id) -> py::object {
        const Seq* q = s.find(id);
        if (!q) return py::none();
        py::dict d;
        d["prompt_len"] = q->prompt.size();
        d["output"] = q->output;
        d["num_computed"] = q->num_computed;
        d["status"] = static_cast<int>(q->status);
        d["finish"] = static_cast<int>(q->finish);
        d["slot"] = q->slot;
        d["num_cached_tokens"] = q->num_cached_tokens;
        d["num_preemptions"] = q->num_preemptions;
        d["arrival_s"] = q->arrival_s;
        d["first_token_s"] = q->first_token_s;
        d["last_token_s"] = q->last_token_s;
        return d;
      })
      .def_property_readonly("prefix_queries", &Scheduler::prefix_queries)
      .def_property_readonly("prefix_hits", &Scheduler::prefix_hits)
      .def_property_readonly("prefix_hit_tokens", &Scheduler::prefix_hit_tokens)
      .def_property_readonly("num_free_blocks", [](Scheduler& s) { return s.kv().num_free_blocks(); })
      .def("kv_usage", [](Scheduler& s) { return s.kv().usage(); });
}
