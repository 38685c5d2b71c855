// HTTP/1.1 server on POSIX sockets for the native OpenAI-compatible API.
//
// One thread accepts; each connection is served on its own thread (keep-alive for plain responses;
// a streamed response (server-sent events) is close-delimited). Requests carry a Content-Length body
// (chunked request bodies are refused with 411), `Expect: 100-continue` is answered, and every
// response carries permissive CORS headers; OPTIONS pre-flights are answered without a handler.
// Replaces the reference's cpp-httplib server (src/server/http_server.cpp:316-449), which is fetched
// from the network at configure time.
#pragma once
#include <atomic>
#include <condition_variable>
#include <functional>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <thread>
#include <utility>
#include <vector>

namespace vmc::http {

struct Request {
  std::string method, target, path, query, version;
  std::vector<std::pair<std::string, std::string>> headers;  // names in lower case
  std::string body;
  std::string header(const std::string& lower_name) const;
};

class Responder {
 public:
  explicit Responder(int fd) : fd_(fd) {}
  // A complete response. Returns false if the client is gone.
  bool send(int status, const std::string& content_type, const std::string& body,
            const std::vector<std::pair<std::string, std::string>>& extra = {});
  // Starts a close-delimited streamed response; write() appends to it.
  bool begin_stream(int status, const std::string& content_type);
  bool write(const std::string& data);
  // True once the peer has closed its side (checked without blocking).
  bool client_gone() const;
  bool responded() const { return responded_; }
  bool streaming() const { return streaming_; }
  void set_keep_alive(bool k) { keep_alive_ = k; }
  bool keep_alive() const { return keep_alive_ && !streaming_; }

 private:
  bool write_all(const char* p, size_t n);
  int fd_;
  bool responded_ = false, streaming_ = false, keep_alive_ = true, broken_ = false;
};

using Handler = std::function<void(const Request&, Responder&)>;

const char* status_text(int status);

class Server {
 public:
  Server() = default;
  ~Server();
  Server(const Server&) = delete;
  Server& operator=(const Server&) = delete;

  void route(const std::string& method, const std::string& path, Handler h);
  void set_max_body_bytes(size_t n) { max_body_ = n; }
  void set_read_timeout_ms(int ms) { read_timeout_ms_ = ms; }
  void set_max_connections(int n) { max_conns_ = n; }

  // Binds and listens; returns the bound port (port 0 picks a free one).
  int listen(const std::string& host, int port);
  // Accept loop on the calling thread until stop().
  void serve_forever();
  // Accept loop on a background thread.
  void start();
  // Stops accepting, shuts the open connections down and waits (bounded) for their threads.
  void stop();
  int active_connections() const { return active_.load(); }

 private:
  void handle(int fd);
  bool read_request(int fd, std::string& carry, Request& req, int& err_status);
  void dispatch(const Request& req, Responder& res);

  std::map<std::pair<std::string, std::string>, Handler> routes_;
  std::set<std::string> paths_;
  int listen_fd_ = -1;
  std::atomic<bool> stopping_{false};
  std::atomic<int> active_{0};
  std::thread acceptor_;
  std::mutex mu_;
  std::condition_variable cv_;
  std::set<int> open_fds_;
  size_t max_body_ = 64u << 20;
  int read_timeout_ms_ = 60000;
  int max_conns_ = 512;
};

}  // namespace vmc::http
