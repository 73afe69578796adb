#include "shm_channel.h"

#include <fcntl.h>
#include <pybind11/stl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <atomic>
#include <chrono>
#include <cstring>
#include <stdexcept>
#include <string>
#include <thread>

namespace py = pybind11;

namespace swift {

constexpr int kMaxReaders = 64;
constexpr uint64_t kMagic = 0x5357494654434831ull;  // "SWIFTCH1"

struct alignas(64) ChannelHeader {
  uint64_t magic;
  uint64_t num_slots;
  uint64_t slot_bytes;
  uint64_t num_readers;
  std::atomic<uint64_t> write_seq;  // messages published
  std::atomic<uint64_t> closed;
  alignas(64) std::atomic<uint64_t> read_seq[kMaxReaders];
  alignas(64) std::atomic<int64_t> heartbeat_ns[kMaxReaders + 1];  // [0] = writer
};

struct SlotHeader {
  std::atomic<uint64_t> seq;
  uint64_t len;
};

static int64_t now_ns() {
  using namespace std::chrono;
  return duration_cast<nanoseconds>(steady_clock::now().time_since_epoch()).count();
}

class TimeoutError : public std::runtime_error {
 public:
  using std::runtime_error::runtime_error;
};
class PeerDiedError : public std::runtime_error {
 public:
  using std::runtime_error::runtime_error;
};

class ShmChannel {
 public:
  // create=true: make (or truncate) the segment; readers attach with create=false.
  ShmChannel(const std::string& name, bool create, int num_readers, int reader_index,
             size_t num_slots, size_t slot_bytes)
      : name_(name), owner_(create), reader_(reader_index) {
    if (num_readers > kMaxReaders) throw std::invalid_argument("too many readers");
    int fd;
    if (create) {
      shm_unlink(name.c_str());
      fd = shm_open(name.c_str(), O_CREAT | O_RDWR, 0600);
    } else {
      fd = shm_open(name.c_str(), O_RDWR, 0600);
    }
    if (fd < 0) throw std::runtime_error("shm_open failed for " + name);
    if (create) {
      size_ = sizeof(ChannelHeader) + num_slots * (sizeof(SlotHeader) + slot_bytes);
      if (ftruncate(fd, static_cast<off_t>(size_)) != 0) {
        ::close(fd);
        throw std::runtime_error("ftruncate failed for " + name);
      }
    } else {
      struct stat st;
      fstat(fd, &st);
      size_ = static_cast<size_t>(st.st_size);
      if (size_ < sizeof(ChannelHeader)) {
        ::close(fd);
        throw std::runtime_error("channel " + name + " not initialised yet");
      }
    }
    base_ = static_cast<uint8_t*>(mmap(nullptr, size_, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0));
    ::close(fd);
    if (base_ == MAP_FAILED) throw std::runtime_error("mmap failed for " + name);
    hdr_ = reinterpret_cast<ChannelHeader*>(base_);
    if (create) {
      std::memset(base_, 0, size_);
      hdr_->num_slots = num_slots;
      hdr_->slot_bytes = slot_bytes;
      hdr_->num_readers = static_cast<uint64_t>(num_readers);
      hdr_->heartbeat_ns[0].store(now_ns());
      std::atomic_thread_fence(std::memory_order_release);
      reinterpret_cast<std::atomic<uint64_t>*>(&hdr_->magic)->store(kMagic, std::memory_order_release);
    } else {
      if (reinterpret_cast<std::atomic<uint64_t>*>(&hdr_->magic)->load(std::memory_order_acquire) != kMagic)
        throw std::runtime_error("channel " + name + " not initialised yet");
      if (reader_ < 0 || reader_ >= static_cast<int>(hdr_->num_readers))
        throw std::invalid_argument("reader index out of range");
      next_ = hdr_->read_seq[reader_].load();
      hdr_->heartbeat_ns[reader_ + 1].store(now_ns());
    }
  }
  ~ShmChannel() {
    if (base_ && base_ != MAP_FAILED) munmap(base_, size_);
    if (owner_) shm_unlink(name_.c_str());
  }

  uint64_t slot_bytes() const { return hdr_->slot_bytes; }

  void beat() { hdr_->heartbeat_ns[owner_ ? 0 : reader_ + 1].store(now_ns(), std::memory_order_relaxed); }

  // Seconds since the given party last stamped its heartbeat (party 0 =
  // writer); -1 if it never has (a worker still loading its weights).
  double heartbeat_age(int party) const {
    const int64_t t = hdr_->heartbeat_ns[party].load(std::memory_order_relaxed);
    if (t == 0) return -1.0;
    return (now_ns() - t) * 1e-9;
  }

  void publish(const char* data, size_t len, double timeout) {
    if (!owner_) throw std::logic_error("only the creating rank publishes");
    if (len > hdr_->slot_bytes) throw std::invalid_argument("message larger than a slot");
    uint64_t seq = hdr_->write_seq.load(std::memory_order_relaxed);
    // wait until every reader consumed the message that used this slot before
    int64_t deadline = now_ns() + static_cast<int64_t>(timeout * 1e9);
    for (int spins = 0;; ++spins) {
      uint64_t slowest = UINT64_MAX;
      for (uint64_t r = 0; r < hdr_->num_readers; ++r)
        slowest = std::min(slowest, hdr_->read_seq[r].load(std::memory_order_acquire));
      if (hdr_->num_readers == 0 || seq < slowest + hdr_->num_slots) break;
      if (now_ns() > deadline) throw TimeoutError("control channel: a worker stopped reading");
      if (spins > 1000) std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
    SlotHeader* s = slot(seq);
    std::memcpy(reinterpret_cast<uint8_t*>(s) + sizeof(SlotHeader), data, len);
    s->len = len;
    s->seq.store(seq + 1, std::memory_order_release);
    hdr_->write_seq.store(seq + 1, std::memory_order_release);
    beat();
  }

  // Returns the next message, or throws TimeoutError / PeerDiedError.
  std::string receive(double timeout, double peer_timeout) {
    if (owner_) throw std::logic_error("the writer does not receive");
    int64_t start = now_ns();
    int64_t deadline = start + static_cast<int64_t>(timeout * 1e9);
    SlotHeader* s = slot(next_);
    for (int spins = 0;; ++spins) {
      if (s->seq.load(std::memory_order_acquire) == next_ + 1) break;
      if (hdr_->closed.load(std::memory_order_acquire))
        throw PeerDiedError("control channel closed by the engine");
      if ((spins & 1023) == 0) {
        beat();
        if (peer_timeout > 0 && heartbeat_age(0) > peer_timeout)
          throw PeerDiedError("engine heartbeat lost");
        if (timeout >= 0 && now_ns() > deadline)
          throw TimeoutError("control channel: no message before the deadline");
        {
          py::gil_scoped_acquire gil;
          if (PyErr_CheckSignals() != 0) throw py::error_already_set();
        }
      }
      if (spins > 2000) std::this_thread::sleep_for(std::chrono::microseconds(spins > 200000 ? 200 : 5));
    }
    size_t len = s->len;
    std::string out(reinterpret_cast<char*>(s) + sizeof(SlotHeader), len);
    ++next_;
    hdr_->read_seq[reader_].store(next_, std::memory_order_release);
    return out;
  }

  void close() { hdr_->closed.store(1, std::memory_order_release); }
  bool closed() const { return hdr_->closed.load(std::memory_order_acquire) != 0; }

  py::bytes receive_py(double timeout, double peer_timeout) {
    std::string out;
    {
      py::gil_scoped_release nogil;
      out = receive(timeout, peer_timeout);
    }
    return py::bytes(out);
  }

 private:
  SlotHeader* slot(uint64_t seq) const {
    size_t stride = sizeof(SlotHeader) + hdr_->slot_bytes;
    return reinterpret_cast<SlotHeader*>(base_ + sizeof(ChannelHeader) +
                                         (seq % hdr_->num_slots) * stride);
  }
  std::string name_;
  bool owner_;
  int reader_;
  uint8_t* base_ = nullptr;
  size_t size_ = 0;
  ChannelHeader* hdr_ = nullptr;
  uint64_t next_ = 0;
};

}  // namespace swift

void bind_shm_channel(py::module_& m) {
  using namespace swift;
  static py::exception<TimeoutError> timeout_exc(m, "ChannelTimeoutError", PyExc_TimeoutError);
  static py::exception<PeerDiedError> died_exc(m, "PeerDiedError", PyExc_RuntimeError);
  py::register_exception_translator([](std::exception_ptr p) {
    try {
      if (p) std::rethrow_exception(p);
    } catch (const TimeoutError& e) {
      PyErr_SetString(timeout_exc.ptr(), e.what());
    } catch (const PeerDiedError& e) {
      PyErr_SetString(died_exc.ptr(), e.what());
    }
  });
  py::class_<ShmChannel>(m, "ShmChannel")
      .def(py::init<const std::string&, bool, int, int, size_t, size_t>(), py::arg("name"),
           py::arg("create"), py::arg("num_readers") = 0, py::arg("reader_index") = -1,
           py::arg("num_slots") = 8, py::arg("slot_bytes") = 1 << 20)
      .def("publish",
           [](ShmChannel& c, py::bytes data, double timeout) {
             char* p;
             py::ssize_t n;
             PYBIND11_BYTES_AS_STRING_AND_SIZE(data.ptr(), &p, &n);
             std::string copy(p, static_cast<size_t>(n));
             py::gil_scoped_release nogil;
             c.publish(copy.data(), copy.size(), timeout);
           },
           py::arg("data"), py::arg("timeout") = 30.0)
      .def("receive", &ShmChannel::receive_py, py::arg("timeout") = -1.0,
           py::arg("peer_timeout") = 0.0)
      .def("beat", &ShmChannel::beat)
      .def("heartbeat_age", &ShmChannel::heartbeat_age)
      .def("close", &ShmChannel::close)
      .def_property_readonly("closed", &ShmChannel::closed)
      .def_property_readonly("slot_bytes", &ShmChannel::slot_bytes);
}
