// HTTP/1.1 server (see http.hpp).
#include "http.hpp"

#include <arpa/inet.h>
#include <netdb.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <sys/socket.h>
#include <unistd.h>

#include <cerrno>
#include <chrono>
#include <cstring>
#include <stdexcept>

namespace vmc::http {

namespace {

const char* const kCors =
    "Access-Control-Allow-Origin: *\r\n"
    "Access-Control-Allow-Methods: GET, POST, OPTIONS\r\n"
    "Access-Control-Allow-Headers: *\r\n";

std::string lower(std::string s) {
  for (char& c : s)
    if (c >= 'A' && c <= 'Z') c = static_cast<char>(c - 'A' + 'a');
  return s;
}

std::string trim(const std::string& s) {
  const size_t b = s.find_first_not_of(" \t");
  if (b == std::string::npos) return "";
  return s.substr(b, s.find_last_not_of(" \t") - b + 1);
}

}  // namespace

const char* status_text(int s) {
  switch (s) {
    case 100: return "Continue";
    case 200: return "OK";
    case 204: return "No Content";
    case 400: return "Bad Request";
    case 404: return "Not Found";
    case 405: return "Method Not Allowed";
    case 408: return "Request Timeout";
    case 411: return "Length Required";
    case 413: return "Payload Too Large";
    case 431: return "Request Header Fields Too Large";
    case 500: return "Internal Server Error";
    case 503: return "Service Unavailable";
    default: return "Unknown";
  }
}

std::string Request::header(const std::string& name) const {
  for (const auto& h : headers)
    if (h.first == name) return h.second;
  return "";
}

bool Responder::write_all(const char* p, size_t n) {
  if (broken_) return false;
  while (n > 0) {
    const ssize_t w = ::send(fd_, p, n, MSG_NOSIGNAL);
    if (w < 0) {
      if (errno == EINTR) continue;
      broken_ = true;
      return false;
    }
    p += w;
    n -= static_cast<size_t>(w);
  }
  return true;
}

bool Responder::send(int status, const std::string& content_type, const std::string& body,
                     const std::vector<std::pair<std::string, std::string>>& extra) {
  if (responded_) return false;
  responded_ = true;
  std::string h = "HTTP/1.1 " + std::to_string(status) + " " + status_text(status) + "\r\n";
  if (!content_type.empty()) h += "Content-Type: " + content_type + "\r\n";
  h += "Content-Length: " + std::to_string(body.size()) + "\r\n";
  h += keep_alive_ ? "Connection: keep-alive\r\n" : "Connection: close\r\n";
  h += kCors;
  for (const auto& e : extra) h += e.first + ": " + e.second + "\r\n";
  h += "\r\n";
  h += body;
  return write_all(h.data(), h.size());
}

bool Responder::begin_stream(int status, const std::string& content_type) {
  if (responded_) return false;
  responded_ = streaming_ = true;
  std::string h = "HTTP/1.1 " + std::to_string(status) + " " + status_text(status) + "\r\n";
  h += "Content-Type: " + content_type + "\r\nCache-Control: no-cache\r\nConnection: close\r\n";
  h += kCors;
  h += "\r\n";
  return write_all(h.data(), h.size());
}

bool Responder::write(const std::string& data) { return streaming_ && write_all(data.data(), data.size()); }

bool Responder::client_gone() const {
  if (broken_) return true;
  pollfd p{fd_, static_cast<short>(POLLIN | POLLRDHUP), 0};
  if (poll(&p, 1, 0) <= 0) return false;
  if (p.revents & (POLLRDHUP | POLLHUP | POLLERR)) return true;
  if (p.revents & POLLIN) {
    char c;
    const ssize_t r = recv(fd_, &c, 1, MSG_PEEK | MSG_DONTWAIT);
    return r == 0;
  }
  return false;
}

Server::~Server() { stop(); }

void Server::route(const std::string& method, const std::string& path, Handler h) {
  routes_[{method, path}] = std::move(h);
  paths_.insert(path);
}

int Server::listen(const std::string& host, int port) {
  addrinfo hints{};
  hints.ai_family = AF_UNSPEC;
  hints.ai_socktype = SOCK_STREAM;
  hints.ai_flags = AI_PASSIVE | AI_NUMERICSERV;
  addrinfo* res = nullptr;
  const std::string ps = std::to_string(port);
  if (getaddrinfo(host.empty() ? nullptr : host.c_str(), ps.c_str(), &hints, &res) != 0 || !res)
    throw std::runtime_error("http: cannot resolve " + host);
  int fd = -1;
  for (addrinfo* a = res; a; a = a->ai_next) {
    fd = socket(a->ai_family, a->ai_socktype, a->ai_protocol);
    if (fd < 0) continue;
    int one = 1;
    setsockopt(fd, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
    if (bind(fd, a->ai_addr, a->ai_addrlen) == 0 && ::listen(fd, 256) == 0) break;
    close(fd);
    fd = -1;
  }
  freeaddrinfo(res);
  if (fd < 0) throw std::runtime_error("http: cannot listen on " + host + ":" + ps + ": " + strerror(errno));
  listen_fd_ = fd;
  sockaddr_storage ss{};
  socklen_t len = sizeof(ss);
  getsockname(fd, reinterpret_cast<sockaddr*>(&ss), &len);
  if (ss.ss_family == AF_INET) return ntohs(reinterpret_cast<sockaddr_in*>(&ss)->sin_port);
  return ntohs(reinterpret_cast<sockaddr_in6*>(&ss)->sin6_port);
}

void Server::serve_forever() {
  if (listen_fd_ < 0) throw std::runtime_error("http: listen() first");
  while (!stopping_.load()) {
    pollfd p{listen_fd_, POLLIN, 0};
    const int r = poll(&p, 1, 200);
    if (r <= 0) continue;
    const int fd = accept(listen_fd_, nullptr, nullptr);
    if (fd < 0) continue;
    if (active_.load() >= max_conns_) {
      Responder res(fd);
      res.set_keep_alive(false);
      res.send(503, "application/json",
               "{\"error\": {\"message\": \"too many connections\", \"type\": \"server_error\", \"code\": 503}}");
      close(fd);
      continue;
    }
    {
      std::lock_guard<std::mutex> lk(mu_);
      open_fds_.insert(fd);
      ++active_;
    }
    std::thread([this, fd] {
      handle(fd);
      std::lock_guard<std::mutex> lk(mu_);
      open_fds_.erase(fd);
      close(fd);
      --active_;
      cv_.notify_all();
    }).detach();
  }
}

void Server::start() {
  acceptor_ = std::thread([this] { serve_forever(); });
}

void Server::stop() {
  if (stopping_.exchange(true)) return;
  if (acceptor_.joinable()) acceptor_.join();
  if (listen_fd_ >= 0) {
    close(listen_fd_);
    listen_fd_ = -1;
  }
  std::unique_lock<std::mutex> lk(mu_);
  for (int fd : open_fds_) shutdown(fd, SHUT_RDWR);
  cv_.wait_for(lk, std::chrono::seconds(10), [this] { return active_.load() == 0; });
}

bool Server::read_request(int fd, std::string& carry, Request& req, int& err) {
  err = 0;
  size_t head_end;
  char buf[16384];
  for (;;) {
    head_end = carry.find("\r\n\r\n");
    if (head_end != std::string::npos) break;
    if (carry.size() > 65536) {
      err = 431;
      return false;
    }
    const ssize_t r = recv(fd, buf, sizeof(buf), 0);
    if (r == 0) return false;  // closed between requests
    if (r < 0) {
      if (errno == EINTR) continue;
      if ((errno == EAGAIN || errno == EWOULDBLOCK) && !carry.empty()) err = 408;
      return false;
    }
    carry.append(buf, static_cast<size_t>(r));
  }
  const std::string head = carry.substr(0, head_end);
  carry.erase(0, head_end + 4);
  size_t eol = head.find("\r\n");
  const std::string line = head.substr(0, eol);
  const size_t s1 = line.find(' '), s2 = line.rfind(' ');
  if (s1 == std::string::npos || s2 == s1) {
    err = 400;
    return false;
  }
  req.method = line.substr(0, s1);
  req.target = line.substr(s1 + 1, s2 - s1 - 1);
  req.version = line.substr(s2 + 1);
  const size_t q = req.target.find('?');
  req.path = req.target.substr(0, q);
  req.query = q == std::string::npos ? "" : req.target.substr(q + 1);
  req.headers.clear();
  while (eol != std::string::npos) {
    const size_t b = eol + 2;
    eol = head.find("\r\n", b);
    const std::string h = head.substr(b, eol == std::string::npos ? std::string::npos : eol - b);
    const size_t c = h.find(':');
    if (c == std::string::npos) continue;
    req.headers.emplace_back(lower(trim(h.substr(0, c))), trim(h.substr(c + 1)));
  }
  if (!req.header("transfer-encoding").empty()) {
    err = 411;
    return false;
  }
  size_t len = 0;
  const std::string cl = req.header("content-length");
  if (!cl.empty()) {
    char* end = nullptr;
    const unsigned long long v = strtoull(cl.c_str(), &end, 10);
    if (!end || *end != '\0') {
      err = 400;
      return false;
    }
    if (v > max_body_) {
      err = 413;
      return false;
    }
    len = static_cast<size_t>(v);
  }
  if (len > carry.size() && lower(req.header("expect")) == "100-continue") {
    const char* cont = "HTTP/1.1 100 Continue\r\n\r\n";
    ::send(fd, cont, strlen(cont), MSG_NOSIGNAL);
  }
  while (carry.size() < len) {
    const ssize_t r = recv(fd, buf, sizeof(buf), 0);
    if (r <= 0) {
      if (r < 0 && errno == EINTR) continue;
      err = r < 0 ? 408 : 0;
      return false;
    }
    carry.append(buf, static_cast<size_t>(r));
  }
  req.body = carry.substr(0, len);
  carry.erase(0, len);
  return true;
}

void Server::dispatch(const Request& req, Responder& res) {
  if (req.method == "OPTIONS") {
    res.send(204, "", "");
    return;
  }
  auto it = routes_.find({req.method, req.path});
  if (it == routes_.end()) {
    const bool known = paths_.count(req.path) != 0;
    const int st = known ? 405 : 404;
    res.send(st, "application/json",
             std::string("{\"error\": {\"message\": \"") + (known ? "method not allowed" : "not found") +
                 "\", \"type\": \"invalid_request_error\", \"code\": " + std::to_string(st) + "}}");
    return;
  }
  try {
    it->second(req, res);
  } catch (const std::exception& e) {
    if (!res.responded()) {
      std::string msg = e.what();
      for (char& c : msg)
        if (c == '"' || c == '\\' || static_cast<unsigned char>(c) < 0x20) c = ' ';
      res.send(500, "application/json",
               "{\"error\": {\"message\": \"" + msg + "\", \"type\": \"server_error\", \"code\": 500}}");
    }
  }
  if (!res.responded()) res.send(500, "application/json", "{\"error\": {\"message\": \"no response\", \"code\": 500}}");
}

void Server::handle(int fd) {
  int one = 1;
  setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
  timeval tv{read_timeout_ms_ / 1000, (read_timeout_ms_ % 1000) * 1000};
  setsockopt(fd, SOL_SOCKET, SO_RCVTIMEO, &tv, sizeof(tv));
  std::string carry;
  while (!stopping_.load()) {
    Request req;
    int err = 0;
    if (!read_request(fd, carry, req, err)) {
      if (err) {
        Responder res(fd);
        res.set_keep_alive(false);
        res.send(err, "application/json",
                 "{\"error\": {\"message\": \"" + std::string(status_text(err)) +
                     "\", \"type\": \"invalid_request_error\", \"code\": " + std::to_string(err) + "}}");
      }
      return;
    }
    Responder res(fd);
    const std::string conn = lower(req.header("connection"));
    const bool keep = req.version == "HTTP/1.1" ? conn != "close" : conn == "keep-alive";
    res.set_keep_alive(keep);
    dispatch(req, res);
    if (!res.keep_alive()) return;
  }
}

}  // namespace vmc::http
