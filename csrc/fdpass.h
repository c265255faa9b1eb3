// File-descriptor exchange between processes of one node.
//
// An exporter serves a fixed list of descriptors on an abstract-namespace
// Unix socket; an importer connects, names an index and receives a duplicate
// through SCM_RIGHTS.  This replaces the reference's pidfd_getfd import
// (sge_write/csrc/storage.hpp:165-178, deepep/csrc/kernels/comm/symmetric.hpp:229-252),
// which requires ptrace permission over the exporter; likewise the server
// answers only peers of its own user id (SO_PEERCRED).
#pragma once

#include <atomic>
#include <string>
#include <thread>
#include <vector>

namespace engram {

class FdServer {
  public:
    // `name` becomes "\0<name>" in the abstract namespace.  The descriptors are
    // borrowed: the caller keeps them open while the server runs.
    FdServer(const std::string &name, std::vector<int> fds);
    ~FdServer();
    FdServer(const FdServer &) = delete;
    FdServer &operator=(const FdServer &) = delete;

    void stop() noexcept;
    const std::string &name() const { return name_; }
    long served() const { return served_.load(); }
    long rejected() const { return rejected_.load(); }  // connections from other users

  private:
    void loop();
    std::string name_;
    std::vector<int> fds_;
    int listen_fd_ = -1;
    std::atomic<bool> stop_{false};
    std::atomic<long> served_{0}, rejected_{0};
    std::thread thread_;
};

// Connects to the server `name` (retrying until `timeout_s`), requests
// descriptor `index` and returns the received duplicate.  Throws on failure.
int fetch_fd(const std::string &name, int index, double timeout_s = 30.0);

} // namespace engram
