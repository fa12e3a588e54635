// Native runtime pieces of cascadia_b200 (module `_runtime`, no CUDA):
//
//  * TCP activation transport between pipeline stages.  Wire format (big
//    endian) as the reference's cascadia-transport crate
//    (crates/cascadia-transport/src/lib.rs:1-16): a 20-byte header
//    [payload_len][dtype][dim0][dim1][dim2] followed by the row-major payload;
//    dtype codes 0=f32 1=f16 2=i8 3=i32 4=i64 (we add 5=bf16 for GPU stages).
//    Caps: 256 MiB per tensor, 64 KiB per raw control read.  Sockets get
//    TCP_NODELAY + keepalive.  Every receive has a deadline; the first byte of
//    a frame may wait up to the idle ceiling, the rest of the frame must
//    arrive within the per-frame timeout.  Errors carry a kind so Python can
//    classify them as connection-fatal (closed / reset / timeout).
//  * Paged-KV block allocator with reference counts (prefix sharing).
//
// The blocking calls release the GIL.
#include <arpa/inet.h>
#include <fcntl.h>
#include <netdb.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <sys/socket.h>
#include <unistd.h>

#include <atomic>
#include <cerrno>
#include <chrono>
#include <cstring>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace py = pybind11;

namespace cbnative {

constexpr size_t kHeader = 20;
constexpr uint64_t kMaxTensorBytes = 256ull * 1024 * 1024;
constexpr size_t kMaxRawBytes = 64 * 1024;

// Transport error with a machine-readable kind.
struct TransportError : std::runtime_error {
  std::string kind;  // closed | reset | timeout | idle_ceiling | protocol | io
  TransportError(const std::string& k, const std::string& msg)
      : std::runtime_error(msg), kind(k) {}
};

static double now_s() {
  return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch())
      .count();
}

static void tune_socket(int fd) {
  int one = 1;
  setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
  setsockopt(fd, SOL_SOCKET, SO_KEEPALIVE, &one, sizeof(one));
#ifdef TCP_KEEPIDLE
  int idle = 30, intvl = 15;
  setsockopt(fd, IPPROTO_TCP, TCP_KEEPIDLE, &idle, sizeof(idle));
  setsockopt(fd, IPPROTO_TCP, TCP_KEEPINTVL, &intvl, sizeof(intvl));
#endif
}

class Link {
 public:
  explicit Link(int fd, double timeout_s, double idle_ceiling_s)
      : fd_(fd), timeout_(timeout_s), idle_(idle_ceiling_s) {
    tune_socket(fd_);
  }
  ~Link() { close(); }

  void close() {
    int fd = fd_.exchange(-1);
    if (fd >= 0) {
      ::shutdown(fd, SHUT_RDWR);
      ::close(fd);
    }
  }
  bool is_open() const { return fd_.load() >= 0; }

  // Send a tensor frame.  `data` is any buffer (bytes, memoryview, numpy).
  void send_tensor(py::buffer data, uint32_t dtype, std::vector<uint32_t> shape) {
    py::buffer_info bi = data.request();
    const uint64_t nbytes = (uint64_t)bi.size * (uint64_t)bi.itemsize;
    if (nbytes > kMaxTensorBytes)
      throw TransportError("protocol", "tensor exceeds 256 MiB wire limit");
    while (shape.size() < 3) shape.insert(shape.begin(), 1u);
    if (shape.size() > 3) throw TransportError("protocol", "tensors up to 3-D only");
    uint8_t hdr[kHeader];
    put_be(hdr + 0, (uint32_t)nbytes);
    put_be(hdr + 4, dtype);
    put_be(hdr + 8, shape[0]);
    put_be(hdr + 12, shape[1]);
    put_be(hdr + 16, shape[2]);
    const uint8_t* p = static_cast<const uint8_t*>(bi.ptr);
    {
      py::gil_scoped_release nogil;
      write_all(hdr, kHeader);
      write_all(p, nbytes);
    }
    sent_bytes_ += kHeader + nbytes;
  }

  // Receive one tensor frame: (dtype, [d0, d1, d2], bytes).  `first_byte_s`
  // bounds the wait for the frame to start (idle ceiling when < 0).
  py::tuple recv_tensor(double first_byte_s) {
    uint8_t hdr[kHeader];
    std::string payload;
    uint32_t dtype, d0, d1, d2;
    {
      py::gil_scoped_release nogil;
      const double start_wait = first_byte_s < 0 ? idle_ : first_byte_s;
      read_exact(hdr, 1, start_wait, first_byte_s < 0 ? 1 : 2);
      const double deadline = now_s() + timeout_;
      read_exact_until(hdr + 1, kHeader - 1, deadline);
      const uint32_t n = get_be(hdr);
      dtype = get_be(hdr + 4);
      d0 = get_be(hdr + 8);
      d1 = get_be(hdr + 12);
      d2 = get_be(hdr + 16);
      if (n > kMaxTensorBytes) throw TransportError("protocol", "frame exceeds 256 MiB");
      payload.resize(n);
      read_exact_until(reinterpret_cast<uint8_t*>(&payload[0]), n, deadline);
      recv_bytes_ += kHeader + n;
    }
    return py::make_tuple(dtype, std::vector<uint32_t>{d0, d1, d2},
                          py::bytes(payload.data(), payload.size()));
  }

  void send_raw(py::bytes b) {
    std::string s = b;
    {
      py::gil_scoped_release nogil;
      write_all(reinterpret_cast<const uint8_t*>(s.data()), s.size());
    }
    sent_bytes_ += s.size();
  }

  py::bytes recv_raw(size_t n, double first_byte_s) {
    if (n > kMaxRawBytes) throw TransportError("protocol", "recv_raw exceeds 64 KiB");
    std::string out(n, '\0');
    {
      py::gil_scoped_release nogil;
      if (n > 0) {
        read_exact(reinterpret_cast<uint8_t*>(&out[0]), 1, first_byte_s < 0 ? idle_ : first_byte_s,
                   first_byte_s < 0 ? 1 : 2);
        read_exact_until(reinterpret_cast<uint8_t*>(&out[1]), n - 1, now_s() + timeout_);
      }
    }
    recv_bytes_ += n;
    return py::bytes(out);
  }

  uint64_t sent_bytes() const { return sent_bytes_; }
  uint64_t recv_bytes() const { return recv_bytes_; }

 private:
  static void put_be(uint8_t* p, uint32_t v) {
    p[0] = v >> 24;
    p[1] = v >> 16;
    p[2] = v >> 8;
    p[3] = v;
  }
  static uint32_t get_be(const uint8_t* p) {
    return ((uint32_t)p[0] << 24) | ((uint32_t)p[1] << 16) | ((uint32_t)p[2] << 8) | p[3];
  }

  int fd() const {
    int f = fd_.load();
    if (f < 0) throw TransportError("closed", "socket closed");
    return f;
  }

  void write_all(const uint8_t* p, uint64_t n) {
    while (n > 0) {
      ssize_t w = ::send(fd(), p, n > (1u << 30) ? (1u << 30) : n, MSG_NOSIGNAL);
      if (w < 0) {
        if (errno == EINTR) continue;
        if (errno == EAGAIN || errno == EWOULDBLOCK) {
          wait_fd(POLLOUT, now_s() + timeout_, 0);
          continue;
        }
        throw_errno("send");
      }
      p += w;
      n -= (uint64_t)w;
    }
  }

  // mode: 0 mid-frame deadline (fatal), 1 idle ceiling (fatal), 2 bounded
  // wait for a frame to start (non-fatal: the caller may retry).
  void wait_fd(short ev, double deadline, int mode) {
    for (;;) {
      const double left = deadline - now_s();
      if (left <= 0) {
        if (mode == 1) throw TransportError("idle_ceiling", "frame start exceeded the idle ceiling");
        if (mode == 2) throw TransportError("frame_start_timeout", "no frame started in time");
        throw TransportError("timeout", "recv_exact timed out");
      }
      pollfd pf{fd(), ev, 0};
      int r = ::poll(&pf, 1, (int)std::min(left * 1000.0 + 1, 1000.0));
      if (r < 0) {
        if (errno == EINTR) continue;
        throw_errno("poll");
      }
      if (r > 0) {
        if (pf.revents & (POLLERR | POLLNVAL)) throw TransportError("reset", "connection reset");
        return;
      }
    }
  }

  void read_exact(uint8_t* p, uint64_t n, double wait_s, int mode) {
    read_exact_until(p, n, now_s() + wait_s, mode);
  }

  void read_exact_until(uint8_t* p, uint64_t n, double deadline, int mode = 0) {
    while (n > 0) {
      wait_fd(POLLIN, deadline, mode);
      ssize_t r = ::recv(fd(), p, n, 0);
      if (r == 0) throw TransportError("closed", "socket closed by peer");
      if (r < 0) {
        if (errno == EINTR || errno == EAGAIN || errno == EWOULDBLOCK) continue;
        throw_errno("recv");
      }
      p += r;
      n -= (uint64_t)r;
    }
  }

  [[noreturn]] static void throw_errno(const char* what) {
    const int e = errno;
    std::string msg = std::string(what) + ": " + std::strerror(e);
    if (e == ECONNRESET) throw TransportError("reset", "connection reset: " + msg);
    if (e == EPIPE) throw TransportError("reset", "broken pipe: " + msg);
    if (e == ECONNABORTED) throw TransportError("reset", "connection aborted: " + msg);
    throw TransportError("io", msg);
  }

  std::atomic<int> fd_;
  double timeout_, idle_;
  uint64_t sent_bytes_ = 0, recv_bytes_ = 0;
};

class Server {
 public:
  Server(const std::string& host, int port) {
    fd_ = ::socket(AF_INET, SOCK_STREAM, 0);
    if (fd_ < 0) throw TransportError("io", "socket() failed");
    int one = 1;
    setsockopt(fd_, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
    sockaddr_in a{};
    a.sin_family = AF_INET;
    a.sin_port = htons((uint16_t)port);
    if (inet_pton(AF_INET, host.c_str(), &a.sin_addr) != 1)
      throw TransportError("io", "bad listen address " + host);
    if (::bind(fd_, reinterpret_cast<sockaddr*>(&a), sizeof(a)) < 0)
      throw TransportError("io", std::string("bind: ") + std::strerror(errno));
    if (::listen(fd_, 8) < 0) throw TransportError("io", "listen failed");
    socklen_t len = sizeof(a);
    getsockname(fd_, reinterpret_cast<sockaddr*>(&a), &len);
    port_ = ntohs(a.sin_port);
  }
  ~Server() { close(); }
  int port() const { return port_; }
  void close() {
    if (fd_ >= 0) {
      ::close(fd_);
      fd_ = -1;
    }
  }

  std::unique_ptr<Link> accept(double timeout_s, double frame_timeout, double idle_ceiling) {
    int c = -1;
    {
      py::gil_scoped_release nogil;
      const double deadline = now_s() + timeout_s;
      for (;;) {
        const double left = deadline - now_s();
        if (left <= 0) throw TransportError("timeout", "accept timed out");
        pollfd pf{fd_, POLLIN, 0};
        int r = ::poll(&pf, 1, (int)std::min(left * 1000.0 + 1, 500.0));
        if (r > 0) {
          c = ::accept(fd_, nullptr, nullptr);
          if (c >= 0) break;
        }
      }
    }
    return std::make_unique<Link>(c, frame_timeout, idle_ceiling);
  }

 private:
  int fd_ = -1;
  int port_ = 0;
};

// Dial with retries every 500 ms for up to `total_s` (the downstream stage may
// still be starting; reference: 500 ms / 30 s).
std::unique_ptr<Link> dial(const std::string& host, int port, double total_s,
                              double frame_timeout, double idle_ceiling) {
  int fd = -1;
  {
    py::gil_scoped_release nogil;
    const double deadline = now_s() + total_s;
    for (;;) {
      addrinfo hints{}, *res = nullptr;
      hints.ai_family = AF_INET;
      hints.ai_socktype = SOCK_STREAM;
      if (getaddrinfo(host.c_str(), std::to_string(port).c_str(), &hints, &res) == 0 && res) {
        fd = ::socket(res->ai_family, res->ai_socktype, res->ai_protocol);
        if (fd >= 0 && ::connect(fd, res->ai_addr, res->ai_addrlen) == 0) {
          freeaddrinfo(res);
          break;
        }
        if (fd >= 0) ::close(fd);
        fd = -1;
        freeaddrinfo(res);
      }
      if (now_s() >= deadline)
        throw TransportError("timeout", "connect to " + host + ":" + std::to_string(port) +
                                            " timed out");
      std::this_thread::sleep_for(std::chrono::milliseconds(500));
    }
  }
  return std::make_unique<Link>(fd, frame_timeout, idle_ceiling);
}

// ------------------------------------------------------------- block allocator
class BlockAllocator {
 public:
  explicit BlockAllocator(int n) : n_(n), ref_(n, 0) {
    free_.reserve(n);
    for (int i = n - 1; i >= 0; --i) free_.push_back(i);
  }
  int num_blocks() const { return n_; }
  int num_free() const { return (int)free_.size(); }
  std::vector<int> allocate(int k) {
    if (k > (int)free_.size())
      throw std::runtime_error("KV cache exhausted: need " + std::to_string(k) + " blocks, " +
                               std::to_string(free_.size()) + " free");
    std::vector<int> out(k);
    for (int i = 0; i < k; ++i) {
      out[i] = free_.back();
      free_.pop_back();
      ref_[out[i]] = 1;
    }
    return out;
  }
  void incref(const std::vector<int>& bs) {
    for (int b : bs) {
      check(b);
      ++ref_[b];
    }
  }
  void free(const std::vector<int>& bs) {
    for (int b : bs) {
      check(b);
      if (ref_[b] <= 0) throw std::runtime_error("double free of KV block " + std::to_string(b));
      if (--ref_[b] == 0) free_.push_back(b);
    }
  }
  int refcount(int b) const {
    check(b);
    return ref_[b];
  }

 private:
  void check(int b) const {
    if (b < 0 || b >= n_) throw std::out_of_range("KV block id out of range");
  }
  int n_;
  std::vector<int> ref_;
  std::vector<int> free_;
};

}  // namespace cbnative

PYBIND11_MODULE(_runtime, m) {
  using namespace cbnative;
  m.doc() = "cascadia_b200 native runtime: TCP stage transport, KV block allocator";
  static py::exception<TransportError> exc(m, "TransportError");
  py::register_exception_translator([](std::exception_ptr p) {
    try {
      if (p) std::rethrow_exception(p);
    } catch (const TransportError& e) {
      PyErr_SetString(exc.ptr(), (e.kind + ": " + e.what()).c_str());
    }
  });
  m.attr("HEADER_SIZE") = kHeader;
  m.attr("MAX_TENSOR_BYTES") = kMaxTensorBytes;
  m.attr("MAX_RAW_BYTES") = kMaxRawBytes;
  py::class_<Link>(m, "Link")
      .def("send_tensor", &Link::send_tensor)
      .def("recv_tensor", &Link::recv_tensor, py::arg("first_byte_s") = -1.0)
      .def("send_raw", &Link::send_raw)
      .def("recv_raw", &Link::recv_raw, py::arg("n"), py::arg("first_byte_s") = -1.0)
      .def("close", &Link::close)
      .def_property_readonly("is_open", &Link::is_open)
      .def_property_readonly("sent_bytes", &Link::sent_bytes)
      .def_property_readonly("recv_bytes", &Link::recv_bytes);
  py::class_<Server>(m, "Server")
      .def(py::init<const std::string&, int>())
      .def_property_readonly("port", &Server::port)
      .def("accept", &Server::accept, py::arg("timeout_s") = 30.0,
           py::arg("frame_timeout") = 60.0, py::arg("idle_ceiling") = 900.0)
      .def("close", &Server::close);
  m.def("connect", &cbnative::dial, py::arg("host"), py::arg("port"), py::arg("total_s") = 30.0,
        py::arg("frame_timeout") = 60.0, py::arg("idle_ceiling") = 900.0);
  py::class_<BlockAllocator>(m, "BlockAllocator")
      .def(py::init<int>())
      .def_property_readonly("num_blocks", &BlockAllocator::num_blocks)
      .def_property_readonly("num_free", &BlockAllocator::num_free)
      .def("allocate", &BlockAllocator::allocate)
      .def("incref", &BlockAllocator::incref)
      .def("free", &BlockAllocator::free)
      .def("refcount", &BlockAllocator::refcount);
}
