// Native HTTP/1.1 front end (see http_server.h).
#include "http_server.h"

#include <arpa/inet.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <sys/epoll.h>
#include <sys/eventfd.h>
#include <sys/socket.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <chrono>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <unordered_map>
#include <unordered_set>

namespace py = pybind11;

namespace swift {

namespace {

const char* reason(int status) {
  switch (status) {
    case 200: return "OK";
    case 204: return "No Content";
    case 400: return "Bad Request";
    case 401: return "Unauthorized";
    case 404: return "Not Found";
    case 405: return "Method Not Allowed";
    case 413: return "Payload Too Large";
    case 500: return "Internal Server Error";
    case 503: return "Service Unavailable";
    default: return "Status";
  }
}

std::string lower(std::string s) {
  for (char& c : s) c = static_cast<char>(std::tolower(static_cast<unsigned char>(c)));
  return s;
}

std::string trim(const std::string& s) {
  size_t a = s.find_first_not_of(" \t"), b = s.find_last_not_of(" \t\r");
  return a == std::string::npos ? std::string() : s.substr(a, b - a + 1);
}

std::string json_error(int status, const std::string& msg, const std::string& kind) {
  std::string m;
  for (char c : msg) {
    if (c == '"' || c == '\\') m += '\\';
    m += c;
  }
  return "{\"error\":{\"message\":\"" + m + "\",\"type\":\"" + kind + "\",\"code\":" +
         std::to_string(status) + "}}";
}

}  // namespace

struct Pending {
  int64_t id;
  std::string method, target, body;
};

struct OutMsg {
  int64_t id;
  std::string data;
  bool finish;  // the response is complete: the connection may take the next request
};

struct Conn {
  int fd = -1;
  std::string in, out;
  int64_t req = -1;  // request in flight (-1: idle)
  bool close_after = false;
  bool want_out = false;
  bool keep_alive = true;
};

class HttpServer {
 public:
  HttpServer(const std::string& host, int port, const std::string& api_key, size_t max_body)
      : api_key_(api_key), max_body_(max_body) {
    lfd_ = ::socket(AF_INET, SOCK_STREAM | SOCK_NONBLOCK | SOCK_CLOEXEC, 0);
    if (lfd_ < 0) throw std::runtime_error("socket() failed");
    int one = 1;
    ::setsockopt(lfd_, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
    sockaddr_in a{};
    a.sin_family = AF_INET;
    a.sin_port = htons(static_cast<uint16_t>(port));
    if (::inet_pton(AF_INET, host == "localhost" ? "127.0.0.1" : host.c_str(), &a.sin_addr) != 1) {
      ::close(lfd_);
      throw std::invalid_argument("bad IPv4 host address: " + host);
    }
    if (::bind(lfd_, reinterpret_cast<sockaddr*>(&a), sizeof(a)) != 0 || ::listen(lfd_, 512) != 0) {
      const std::string e = std::strerror(errno);
      ::close(lfd_);
      throw std::runtime_error("bind/listen failed: " + e);
    }
    socklen_t len = sizeof(a);
    ::getsockname(lfd_, reinterpret_cast<sockaddr*>(&a), &len);
    port_ = ntohs(a.sin_port);
    efd_ = ::eventfd(0, EFD_NONBLOCK | EFD_CLOEXEC);
    epfd_ = ::epoll_create1(EPOLL_CLOEXEC);
    add_fd(lfd_, EPOLLIN);
    add_fd(efd_, EPOLLIN);
  }

  ~HttpServer() {
    stop();
    for (auto& kv : conns_) ::close(kv.first);
    ::close(lfd_);
    ::close(efd_);
    ::close(epfd_);
  }

  int port() const { return port_; }

  void start() {
    if (thread_.joinable()) return;
    running_ = true;
    thread_ = std::thread([this] { loop(); });
  }

  void stop() {
    if (!thread_.joinable()) return;
    running_ = false;
    wake();
    thread_.join();
    cv_.notify_all();
  }

  // Next request for the engine: (id, method, target, body) or None.
  py::object poll(double timeout) {
    Pending p;
    {
      py::gil_scoped_release nogil;
      std::unique_lock<std::mutex> lk(mu_);
      auto until = std::chrono::steady_clock::now() +
                   std::chrono::microseconds(static_cast<int64_t>(std::max(0.0, timeout) * 1e6));
      if (!cv_.wait_until(lk, until, [&] { return !inbox_.empty() || !running_; })) {
        return py::none();
      }
      if (inbox_.empty()) return py::none();
      p = std::move(inbox_.front());
      inbox_.pop_front();
    }
    return py::make_tuple(p.id, p.method, p.target, py::bytes(p.body));
  }

  void respond(int64_t id, int status, const std::string& ctype, const std::string& body) {
    std::string h = "HTTP/1.1 " + std::to_string(status) + " " + reason(status) +
                    "\r\nContent-Type: " + ctype + "\r\nContent-Length: " +
                    std::to_string(body.size()) + "\r\nAccess-Control-Allow-Origin: *\r\n\r\n";
    push({id, h + body, true});
  }
  void stream_start(int64_t id) {
    push({id,
          "HTTP/1.1 200 OK\r\nContent-Type: text/event-stream\r\nCache-Control: no-cache\r\n"
          "Transfer-Encoding: chunked\r\nAccess-Control-Allow-Origin: *\r\n\r\n",
          false});
  }
  void stream_send(int64_t id, const std::string& data) {
    if (data.empty()) return;
    char hex[32];
    std::snprintf(hex, sizeof(hex), "%zx\r\n", data.size());
    push({id, std::string(hex) + data + "\r\n", false});
  }
  void stream_end(int64_t id) { push({id, "0\r\n\r\n", true}); }

  bool is_open(int64_t id) {
    std::lock_guard<std::mutex> lk(mu_);
    return open_.count(id) != 0;
  }

  py::dict stats() {
    std::lock_guard<std::mutex> lk(mu_);
    py::dict d;
    d["connections"] = conn_count_;
    d["requests"] = next_id_ - 1;
    d["answered_natively"] = native_answers_;
    d["pending"] = inbox_.size();
    return d;
  }

 private:
  void add_fd(int fd, uint32_t ev) {
    epoll_event e{};
    e.events = ev;
    e.data.fd = fd;
    ::epoll_ctl(epfd_, EPOLL_CTL_ADD, fd, &e);
  }
  void mod_fd(int fd, uint32_t ev) {
    epoll_event e{};
    e.events = ev;
    e.data.fd = fd;
    ::epoll_ctl(epfd_, EPOLL_CTL_MOD, fd, &e);
  }
  void wake() {
    uint64_t one = 1;
    ssize_t r = ::write(efd_, &one, sizeof(one));
    (void)r;
  }
  void push(OutMsg m) {
    {
      std::lock_guard<std::mutex> lk(mu_);
      outbox_.push_back(std::move(m));
    }
    wake();
  }

  void close_conn(int fd) {
    auto it = conns_.find(fd);
    if (it == conns_.end()) return;
    if (it->second.req >= 0) {
      std::lock_guard<std::mutex> lk(mu_);
      open_.erase(it->second.req);
      id_fd_.erase(it->second.req);
    }
    ::epoll_ctl(epfd_, EPOLL_CTL_DEL, fd, nullptr);
    ::close(fd);
    conns_.erase(it);
  }

  // queue bytes on a connection (I/O thread only)
  void send_raw(Conn& c, const std::string& data) {
    c.out += data;
    flush(c);
  }

  void native(Conn& c, int status, const std::string& ctype, const std::string& body,
              const std::string& extra = "") {
    ++native_answers_;
    send_raw(c, "HTTP/1.1 " + std::to_string(status) + " " + reason(status) +
                    "\r\nContent-Type: " + ctype + "\r\nContent-Length: " +
                    std::to_string(body.size()) + "\r\nAccess-Control-Allow-Origin: *\r\n" +
                    extra + "\r\n" + body);
    if (!c.keep_alive) c.close_after = true;
  }

  void flush(Conn& c) {
    while (!c.out.empty()) {
      ssize_t n = ::send(c.fd, c.out.data(), c.out.size(), MSG_NOSIGNAL);
      if (n > 0) {
        c.out.erase(0, static_cast<size_t>(n));
        continue;
      }
      if (n < 0 && (errno == EAGAIN || errno == EWOULDBLOCK)) break;
      c.close_after = true;
      c.out.clear();
      break;
    }
    const bool want = !c.out.empty();
    if (want != c.want_out) {
      c.want_out = want;
      mod_fd(c.fd, EPOLLIN | EPOLLRDHUP | (want ? EPOLLOUT : 0));
    }
  }

  // Parse as many complete requests as the connection has (one in flight).
  void parse(Conn& c) {
    while (c.req < 0 && !c.close_after) {
      size_t he = c.in.find("\r\n\r\n");
      if (he == std::string::npos) {
        if (c.in.size() > 65536) {
          c.keep_alive = false;
          native(c, 400, "application/json", json_error(400, "header too large", "invalid_request_error"));
        }
        return;
      }
      std::string head = c.in.substr(0, he);
      size_t le = head.find("\r\n");
      std::string line = head.substr(0, le);
      size_t s1 = line.find(' '), s2 = line.find(' ', s1 + 1);
      if (s1 == std::string::npos || s2 == std::string::npos) {
        c.keep_alive = false;
        native(c, 400, "application/json", json_error(400, "malformed request line", "invalid_request_error"));
        return;
      }
      std::string method = line.substr(0, s1), target = line.substr(s1 + 1, s2 - s1 - 1);
      std::string version = line.substr(s2 + 1);
      size_t clen = 0;
      std::string auth, conn_hdr;
      size_t pos = le == std::string::npos ? head.size() : le + 2;
      while (pos < head.size()) {
        size_t e = head.find("\r\n", pos);
        if (e == std::string::npos) e = head.size();
        std::string h = head.substr(pos, e - pos);
        size_t colon = h.find(':');
        if (colon != std::string::npos) {
          std::string k = lower(trim(h.substr(0, colon))), v = trim(h.substr(colon + 1));
          if (k == "content-length") clen = static_cast<size_t>(std::strtoull(v.c_str(), nullptr, 10));
          else if (k == "authorization") auth = v;
          else if (k == "connection") conn_hdr = lower(v);
        }
        pos = e + 2;
      }
      c.keep_alive = version == "HTTP/1.1" ? conn_hdr != "close" : conn_hdr == "keep-alive";
      if (clen > max_body_) {
        c.keep_alive = false;
        native(c, 413, "application/json", json_error(413, "request body too large", "invalid_request_error"));
        return;
      }
      if (c.in.size() < he + 4 + clen) return;  // body still arriving
      std::string body = c.in.substr(he + 4, clen);
      c.in.erase(0, he + 4 + clen);
      std::string path = target.substr(0, target.find('?'));
      if (method == "OPTIONS") {
        native(c, 204, "text/plain", "",
               "Access-Control-Allow-Methods: GET, POST, OPTIONS\r\n"
               "Access-Control-Allow-Headers: Content-Type, Authorization\r\n");
        continue;
      }
      if (method == "GET" && (path == "/health" || path == "/v1/health")) {
        native(c, 200, "application/json", "{\"status\":\"ok\"}");
        continue;
      }
      if (!api_key_.empty() && path.rfind("/v1", 0) == 0 && auth != "Bearer " + api_key_) {
        native(c, 401, "application/json",
               json_error(401, "invalid or missing API key", "authentication_error"));
        continue;
      }
      {
        std::lock_guard<std::mutex> lk(mu_);
        const int64_t id = next_id_++;
        c.req = id;
        id_fd_[id] = c.fd;
        open_.insert(id);
        inbox_.push_back({id, method, target, std::move(body)});
      }
      cv_.notify_one();
    }
  }

  void drain_outbox() {
    std::deque<OutMsg> msgs;
    {
      std::lock_guard<std::mutex> lk(mu_);
      msgs.swap(outbox_);
    }
    for (auto& m : msgs) {
      int fd;
      {
        std::lock_guard<std::mutex> lk(mu_);
        auto it = id_fd_.find(m.id);
        if (it == id_fd_.end()) continue;  // client gone
        fd = it->second;
        if (m.finish) {
          id_fd_.erase(it);
          open_.erase(m.id);
        }
      }
      auto ci = conns_.find(fd);
      if (ci == conns_.end()) continue;
      Conn& c = ci->second;
      send_raw(c, m.data);
      if (m.finish) {
        c.req = -1;
        if (!c.keep_alive) c.close_after = true;
        parse(c);  // a pipelined request may already be buffered
      }
      if (c.close_after && c.out.empty()) close_conn(fd);
    }
  }

  void loop() {
    epoll_event evs[128];
    while (running_) {
      int n = ::epoll_wait(epfd_, evs, 128, 100);
      for (int i = 0; i < n; ++i) {
        const int fd = evs[i].data.fd;
        const uint32_t ev = evs[i].events;
        if (fd == lfd_) {
          for (;;) {
            int cfd = ::accept4(lfd_, nullptr, nullptr, SOCK_NONBLOCK | SOCK_CLOEXEC);
            if (cfd < 0) break;
            int one = 1;
            ::setsockopt(cfd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
            Conn c;
            c.fd = cfd;
            conns_.emplace(cfd, std::move(c));
            add_fd(cfd, EPOLLIN | EPOLLRDHUP);
            ++conn_count_;
          }
          continue;
        }
        if (fd == efd_) {
          uint64_t v;
          while (::read(efd_, &v, sizeof(v)) > 0) {
          }
          drain_outbox();
          continue;
        }
        auto it = conns_.find(fd);
        if (it == conns_.end()) continue;
        Conn& c = it->second;
        bool gone = (ev & (EPOLLHUP | EPOLLERR)) != 0;
        if (ev & EPOLLIN) {
          char buf[65536];
          for (;;) {
            ssize_t r = ::recv(fd, buf, sizeof(buf), 0);
            if (r > 0) {
              c.in.append(buf, static_cast<size_t>(r));
              continue;
            }
            if (r == 0) gone = true;
            else if (errno != EAGAIN && errno != EWOULDBLOCK) gone = true;
            break;
          }
        }
        if ((ev & EPOLLRDHUP) && c.in.empty()) gone = true;
        if (gone) {
          close_conn(fd);
          continue;
        }
        if (ev & EPOLLOUT) flush(c);
        parse(c);
        if (c.close_after && c.out.empty()) close_conn(fd);
      }
      drain_outbox();
    }
  }

  std::string api_key_;
  size_t max_body_;
  int lfd_ = -1, efd_ = -1, epfd_ = -1, port_ = 0;
  std::atomic<bool> running_{false};
  std::thread thread_;
  std::unordered_map<int, Conn> conns_;  // I/O thread only
  std::mutex mu_;
  std::condition_variable cv_;
  std::deque<Pending> inbox_;
  std::deque<OutMsg> outbox_;
  std::unordered_map<int64_t, int> id_fd_;
  std::unordered_set<int64_t> open_;
  int64_t next_id_ = 1;
  int64_t conn_count_ = 0, native_answers_ = 0;
};

}  // namespace swift

void bind_http_server(py::module_& m) {
  using swift::HttpServer;
  py::class_<HttpServer>(m, "HttpServer")
      .def(py::init<const std::string&, int, const std::string&, size_t>(), py::arg("host") = "127.0.0.1",
           py::arg("port") = 0, py::arg("api_key") = "", py::arg("max_body") = size_t(16) << 20)
      .def_property_readonly("port", &HttpServer::port)
      .def("start", &HttpServer::start)
      .def("stop", &HttpServer::stop, py::call_guard<py::gil_scoped_release>())
      .def("poll", &HttpServer::poll, py::arg("timeout") = 0.0)
      .def("respond", &HttpServer::respond, py::arg("id"), py::arg("status"),
           py::arg("content_type"), py::arg("body"))
      .def("stream_start", &HttpServer::stream_start)
      .def("stream_send", &HttpServer::stream_send)
      .def("stream_end", &HttpServer::stream_end)
      .def("is_open", &HttpServer::is_open)
      .def("stats", &HttpServer::stats);
}
