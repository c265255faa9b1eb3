// CPU test harnesses: the owner service and descriptor passing without a GPU.
// They drive the same OwnerService and FdServer code the runtime uses, so the
// mailbox sequence rules, error latching and SCM_RIGHTS exchange are tested
// on machines with no GPU.
#include <pybind11/stl.h>

#include <sys/mman.h>
#include <unistd.h>

#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "bindings.h"
#include "driver.h"
#include "fdpass.h"
#include "kernels/params.h"
#include "owner_service.h"
#include "trace.h"

namespace py = pybind11;

namespace engram {

namespace {

class OwnerServiceHarness {
  public:
    OwnerServiceHarness(uint32_t world, uint32_t layers, uint32_t capacity, std::vector<uint8_t> serve)
        : world_(world), layers_(layers), capacity_(capacity), serve_(std::move(serve)),
          headers_(size_t(world) * layers) {
        std::memset(headers_.data(), 0, headers_.size() * sizeof(MailboxHeader));
    }
    ~OwnerServiceHarness() { service_.stop_and_join(); }

    void publish(uint32_t requester, uint32_t layer, uint64_t epoch, uint32_t rows, uint32_t channels) {
        MailboxHeader *h = &headers_.at(size_t(requester) * layers_ + layer);
        __atomic_store_n(&h->rows, rows, __ATOMIC_RELAXED);
        __atomic_store_n(&h->layer, layer, __ATOMIC_RELAXED);
        __atomic_store_n(&h->requester, requester, __ATOMIC_RELAXED);
        __atomic_store_n(&h->channels, channels, __ATOMIC_RELAXED);
        __atomic_store_n(&h->ready, epoch, __ATOMIC_RELEASE);
    }
    void start(int fail_after) {
        OwnerServiceConfig c;
        c.world = world_;
        c.layers = layers_;
        c.capacity = capacity_;
        c.headers = headers_.data();
        c.serve = serve_;
        c.idle_spin_us = 1000;
        c.nap_us = 20;
        fail_after_ = fail_after;
        service_.start(std::move(c), [this](const std::vector<PushTask> &batch) {
            std::lock_guard<std::mutex> lock(mu_);
            for (const auto &t : batch) {
                if (fail_after_ >= 0 && int(launched_.size()) >= fail_after_)
                    throw std::runtime_error("injected launch failure");
                launched_.push_back(t);
            }
        });
    }
    void stop() {
        py::gil_scoped_release release;
        service_.stop_and_join();
    }
    py::list launched() {
        std::lock_guard<std::mutex> lock(mu_);
        py::list out;
        for (const auto &t : launched_)
            out.append(py::make_tuple(t.requester, t.layer, t.rows, t.epoch, t.channels));
        return out;
    }
    std::string error() { return service_.error(); }
    void check() { service_.check(); }
    bool running() const { return service_.running(); }

  private:
    uint32_t world_, layers_, capacity_;
    std::vector<uint8_t> serve_;
    std::vector<MailboxHeader> headers_;
    OwnerService service_;
    std::mutex mu_;
    std::vector<PushTask> launched_;
    int fail_after_ = -1;
};

int memfd_with_bytes(const std::string &data) {
    int fd = memfd_create("engram-test", MFD_CLOEXEC);
    check(fd >= 0, "memfd_create");
    check(ftruncate(fd, off_t(data.size())) == 0, "ftruncate");
    check(pwrite(fd, data.data(), data.size(), 0) == ssize_t(data.size()), "pwrite");
    return fd;
}

py::bytes read_fd_bytes(int fd, size_t n) {
    std::string out(n, '\0');
    check(pread(fd, out.data(), n, 0) == ssize_t(n), "pread");
    return py::bytes(out);
}


} // namespace

void bind_harness(py::module_ &m) {
    py::class_<OwnerServiceHarness>(m, "OwnerServiceHarness")
        .def(py::init<uint32_t, uint32_t, uint32_t, std::vector<uint8_t>>())
        .def("publish", &OwnerServiceHarness::publish)
        .def("start", &OwnerServiceHarness::start, py::arg("fail_after") = -1)
        .def("stop", &OwnerServiceHarness::stop)
        .def("launched", &OwnerServiceHarness::launched)
        .def("error", &OwnerServiceHarness::error)
        .def("check", &OwnerServiceHarness::check)
        .def_property_readonly("running", &OwnerServiceHarness::running);
    py::class_<FdServer>(m, "FdServer")
        .def(py::init<const std::string &, std::vector<int>>())
        .def("stop", &FdServer::stop)
        .def_property_readonly("served", &FdServer::served)
        .def_property_readonly("rejected", &FdServer::rejected);
    m.def("fetch_fd", &fetch_fd, py::arg("name"), py::arg("index"), py::arg("timeout_s") = 30.0);
    m.def("memfd_with_bytes", &memfd_with_bytes);
    m.def("read_fd_bytes", &read_fd_bytes);
}

} // namespace engram
