// vmc_serve_cpu: the native OpenAI server over a host-only step backend.
//
//   vmc_serve_cpu MODEL.gguf [--host 127.0.0.1] [--port 8000] [--model-name NAME] [--max-num-seqs S]
//                 [--max-num-batched-tokens T] [--max-model-len L] [--num-blocks B] [--port-file PATH]
//                 [--step-delay-ms D]
//
// Everything the GPU server runs except the forward: GGUF vocabulary and tokenizer, chat prompts,
// HTTP / SSE, the serving loop with the continuous-batching scheduler and block manager. The step
// backend is a deterministic rule instead of a model: the token after token t at position p is
// (31 t + 7 p + 11) mod V. A client can therefore predict every completion exactly, which makes this
// binary the test bed of the server's request handling, scheduling and streaming (the GPU server in
// vmc_run differs only in its backend).
//
// Two tool modes read one JSON value per stdin line and print one JSON value per line, for checking
// the text pipeline against the Python tokenizer and chat templates:
//   vmc_serve_cpu --tool pre-split FAMILY      a string -> the pieces of pre-tokeniser FAMILY
//   vmc_serve_cpu --tool utf8-stream -         byte chunks [[b, ...], ...] -> the text each chunk
//                                              releases through the streaming UTF-8 decoder
//   vmc_serve_cpu --tool json -                a line -> the document re-serialised, or
//                                              {"error": offset} if it is not valid JSON
//   vmc_serve_cpu --tool render-chat TEMPLATE_FILE
//       {"messages": [...], "add_generation_prompt": b, "enable_thinking": b, "bos": s, "eos": s}
//       -> the chat prompt the server builds with that Jinja template (an empty file: ChatML);
//       TEMPLATE_FILE "-": each line carries its own "template"
#include <atomic>
#include <chrono>
#include <cstdio>
#include <fstream>
#include <iostream>
#include <sstream>
#include <cstring>
#include <stdexcept>
#include <string>
#include <thread>

#include "gguf.hpp"
#include "http.hpp"
#include "json.hpp"
#include "openai.hpp"
#include "serve_loop.hpp"
#include "stop_signals.hpp"
#include "text_tokenizer.hpp"
#include "unicode.hpp"

namespace {

class RuleBackend : public vmc::StepBackend {
 public:
  RuleBackend(vmc::BatchLayout layout, int vocab, int delay_ms) : layout_(layout), vocab_(vocab), delay_ms_(delay_ms) {}
  vmc::BatchLayout layout() const override { return layout_; }
  int vocab() const override { return vocab_; }
  int graph_bucket(int n) const override {  // exercise the padded decode path as the GPU backend does
    int b = 1;
    while (b < n) b *= 2;
    return b <= layout_.max_reqs ? b : 0;
  }
  void step(const int32_t* meta, const vmc::SampleParams*, int S, const vmc::Penalties&, int32_t* tokens,
            float* logprobs) override {
    if (delay_ms_ > 0) std::this_thread::sleep_for(std::chrono::milliseconds(delay_ms_));  // a slower "model"
    const int32_t* ids = meta + layout_.off_input_ids();
    const int32_t* pos = meta + layout_.off_positions();
    const int32_t* row = meta + layout_.off_logits_idx();
    for (int k = 0; k < S; ++k) {
      const int64_t r = row[k];
      if (r < 0 || r >= layout_.max_tokens) throw std::runtime_error("rule backend: sample row out of range");
      tokens[k] = static_cast<int32_t>((31LL * ids[r] + 7LL * pos[r] + 11) % vocab_);
      logprobs[k] = 0.f;
    }
  }

 private:
  vmc::BatchLayout layout_;
  int vocab_, delay_ms_;
};


int run_tool(const std::string& tool, const std::string& arg) {
  using vmc::json::Value;
  std::string tmpl;
  if (tool == "render-chat") {
    if (arg != "-") {
      std::ifstream f(arg);
      if (!f) throw std::runtime_error("cannot read " + arg);
      std::stringstream ss;
      ss << f.rdbuf();
      tmpl = ss.str();
    }
  } else if (tool != "pre-split" && tool != "utf8-stream" && tool != "json") {
    throw std::runtime_error("unknown tool " + tool);
  }
  std::string line;
  while (std::getline(std::cin, line)) {
    if (tool == "json") {  // the parser itself is under test: report a rejection instead of failing
      try {
        std::cout << vmc::json::dump(vmc::json::parse(line)) << "\n";
      } catch (const vmc::json::ParseError& e) {
        std::cout << "{\"error\": " << e.offset() << "}\n";
      }
      continue;
    }
    const Value in = vmc::json::parse(line);
    Value out;
    if (tool == "pre-split") {
      out = Value::array();
      for (const auto& p : vmc::TextTokenizer::pre_split(in.as_string(), arg)) out.push(p);
    } else if (tool == "utf8-stream") {
      out = Value::array();
      std::string buf;
      const auto& chunks = in.as_array();
      for (size_t k = 0; k < chunks.size(); ++k) {
        for (const Value& b : chunks[k].as_array()) buf += static_cast<char>(b.as_int());
        std::string text;
        buf.erase(0, vmc::uni::decode_stream(buf, k + 1 == chunks.size(), text));
        out.push(text);
      }
    } else {
      std::vector<vmc::ChatMessage> msgs;
      for (const Value& m : in.get("messages")->as_array())
        msgs.push_back({m.get_string("role", "user"), m.get_string("content", "")});
      const vmc::ChatTemplate ct(arg == "-" ? in.get_string("template", "") : tmpl, in.get_string("bos", ""),
                                 in.get_string("eos", ""));
      std::string why;
      out = ct.render(msgs, in.get_bool("add_generation_prompt", true), in.get_bool("enable_thinking", true), &why);
      if (!why.empty()) std::cerr << "chat template: " << why << "\n";
    }
    std::cout << vmc::json::dump(out) << "\n";
  }
  std::cout.flush();
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  try {
    if (argc < 2) throw std::runtime_error("usage: vmc_serve_cpu MODEL.gguf [options]");
    if (std::string(argv[1]) == "--tool") {
      if (argc != 4) throw std::runtime_error("usage: vmc_serve_cpu --tool NAME ARG");
      return run_tool(argv[2], argv[3]);
    }
    std::string host = "127.0.0.1", name = "vm_c", port_file;
    int port = 8000, max_seqs = 16, max_batched = 256, max_len = 1024, num_blocks = 0, delay_ms = 0;
    for (int i = 2; i < argc; ++i) {
      const std::string k = argv[i];
      auto val = [&]() -> std::string {
        if (i + 1 >= argc) throw std::runtime_error("missing value for " + k);
        return argv[++i];
      };
      if (k == "--host") host = val();
      else if (k == "--port") port = std::stoi(val());
      else if (k == "--model-name") name = val();
      else if (k == "--max-num-seqs") max_seqs = std::stoi(val());
      else if (k == "--max-num-batched-tokens") max_batched = std::stoi(val());
      else if (k == "--max-model-len") max_len = std::stoi(val());
      else if (k == "--num-blocks") num_blocks = std::stoi(val());
      else if (k == "--port-file") port_file = val();
      else if (k == "--step-delay-ms") delay_ms = std::stoi(val());
      else throw std::runtime_error("unknown option " + k);
    }
    vmc::StopSignals stop;  // before any thread exists
    auto gguf = vmc::GgufFile::open(argv[1]);
    auto tok = vmc::TextTokenizer::from_gguf(*gguf);
    const int max_blocks = (max_len + 15) / 16 + 1;
    vmc::BatchLayout layout{std::max(max_batched, max_seqs), max_seqs, max_blocks};
    RuleBackend be(layout, tok->vocab_size(), delay_ms);
    vmc::ServeConfig sc;
    sc.sched.max_num_seqs = max_seqs;
    sc.sched.max_num_batched_tokens = max_batched;
    sc.sched.max_model_len = max_len;
    sc.num_blocks = num_blocks > 0 ? num_blocks : static_cast<int64_t>(max_seqs) * max_blocks + 1;
    sc.eos_token_ids = tok->eos_ids();
    vmc::ServeLoop loop(sc, be);
    vmc::OpenAIConfig oc;
    oc.model_name = name;
    vmc::OpenAIServer api(loop, *tok, oc);
    vmc::http::Server srv;
    api.install(srv);
    const int bound = srv.listen(host, port);
    fprintf(stderr, "vmc_serve_cpu: listening on %s:%d (chat template: %s)\n", host.c_str(), bound,
            api.chat_template().has_template() ? "jinja" : ("ChatML " + api.chat_template().parse_error()).c_str());
    if (!port_file.empty()) {
      FILE* f = fopen(port_file.c_str(), "w");
      if (!f) throw std::runtime_error("cannot write " + port_file);
      fprintf(f, "%d\n", bound);
      fclose(f);
    }
    srv.start();
    std::atomic<bool> done{false};
    std::thread watcher([&] {
      while (!done.load())
        if (stop.wait(100)) {
          loop.request_stop();
          return;
        }
    });
    loop.run();
    done.store(true);
    watcher.join();
    srv.stop();
    return 0;
  } catch (const std::exception& e) {
    fprintf(stderr, "vmc_serve_cpu: %s\n", e.what());
    return 1;
  }
}
