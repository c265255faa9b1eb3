#include "fdpass.h"

#include <poll.h>
#include <sys/socket.h>
#include <sys/un.h>
#include <unistd.h>

#include <cerrno>
#include <chrono>
#include <cstring>
#include <stdexcept>
#include <thread>

namespace engram {

namespace {

socklen_t make_address(const std::string &name, sockaddr_un *addr) {
    std::memset(addr, 0, sizeof(*addr));
    addr->sun_family = AF_UNIX;
    if (name.size() + 1 > sizeof(addr->sun_path))
        throw std::runtime_error("socket name too long");
    // Abstract namespace: leading NUL, no filesystem entry to clean up.
    std::memcpy(addr->sun_path + 1, name.data(), name.size());
    return socklen_t(offsetof(sockaddr_un, sun_path) + 1 + name.size());
}

bool send_fd(int sock, int fd, char status) {
    char byte = status;
    iovec iov{&byte, 1};
    msghdr msg{};
    msg.msg_iov = &iov;
    msg.msg_iovlen = 1;
    alignas(cmsghdr) char control[CMSG_SPACE(sizeof(int))];
    if (status == 0 && fd >= 0) {
        std::memset(control, 0, sizeof(control));
        msg.msg_control = control;
        msg.msg_controllen = sizeof(control);
        cmsghdr *c = CMSG_FIRSTHDR(&msg);
        c->cmsg_level = SOL_SOCKET;
        c->cmsg_type = SCM_RIGHTS;
        c->cmsg_len = CMSG_LEN(sizeof(int));
        std::memcpy(CMSG_DATA(c), &fd, sizeof(int));
    }
    return sendmsg(sock, &msg, MSG_NOSIGNAL) == 1;
}

} // namespace

FdServer::FdServer(const std::string &name, std::vector<int> fds) : name_(name), fds_(std::move(fds)) {
    listen_fd_ = socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
    if (listen_fd_ < 0)
        throw std::runtime_error("fd server: socket() failed");
    sockaddr_un addr;
    socklen_t len = make_address(name_, &addr);
    if (bind(listen_fd_, reinterpret_cast<sockaddr *>(&addr), len) != 0 || listen(listen_fd_, 64) != 0) {
        int err = errno;
        ::close(listen_fd_);
        listen_fd_ = -1;
        throw std::runtime_error(std::string("fd server: bind/listen failed: ") + std::strerror(err));
    }
    thread_ = std::thread([this] { loop(); });
}

void FdServer::loop() {
    while (!stop_.load(std::memory_order_relaxed)) {
        pollfd p{listen_fd_, POLLIN, 0};
        int ready = poll(&p, 1, 50);
        if (ready <= 0)
            continue;
        int conn = accept4(listen_fd_, nullptr, nullptr, SOCK_CLOEXEC);
        if (conn < 0)
            continue;
        // Abstract socket names are visible to every local user
        // (/proc/net/unix): hand descriptors only to processes of this
        // user, as pidfd_getfd's ptrace check would.
        ucred cred{};
        socklen_t cred_len = sizeof(cred);
        if (getsockopt(conn, SOL_SOCKET, SO_PEERCRED, &cred, &cred_len) != 0 || cred.uid != getuid()) {
            rejected_.fetch_add(1);
            ::close(conn);
            continue;
        }
        // Bounded request read: a client that never sends is dropped.
        pollfd q{conn, POLLIN, 0};
        int32_t index = -1;
        if (poll(&q, 1, 5000) > 0 && recv(conn, &index, sizeof(index), MSG_WAITALL) == sizeof(index)) {
            bool ok = index >= 0 && size_t(index) < fds_.size() && fds_[index] >= 0;
            if (send_fd(conn, ok ? fds_[index] : -1, ok ? 0 : 1) && ok)
                served_.fetch_add(1);
        }
        ::close(conn);
    }
}

void FdServer::stop() noexcept {
    stop_.store(true);
    if (thread_.joinable())
        thread_.join();
    if (listen_fd_ >= 0) {
        ::close(listen_fd_);
        listen_fd_ = -1;
    }
}

FdServer::~FdServer() { stop(); }

int fetch_fd(const std::string &name, int index, double timeout_s) {
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::duration<double>(timeout_s);
    std::string last = "no attempt";
    while (true) {
        int sock = socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
        if (sock < 0)
            throw std::runtime_error("fd client: socket() failed");
        sockaddr_un addr;
        socklen_t len = make_address(name, &addr);
        if (connect(sock, reinterpret_cast<sockaddr *>(&addr), len) == 0) {
            int32_t req = index;
            if (send(sock, &req, sizeof(req), MSG_NOSIGNAL) == sizeof(req)) {
                char status = 1;
                iovec iov{&status, 1};
                msghdr msg{};
                msg.msg_iov = &iov;
                msg.msg_iovlen = 1;
                alignas(cmsghdr) char control[CMSG_SPACE(sizeof(int))];
                msg.msg_control = control;
                msg.msg_controllen = sizeof(control);
                pollfd p{sock, POLLIN, 0};
                if (poll(&p, 1, 10000) > 0 && recvmsg(sock, &msg, MSG_CMSG_CLOEXEC) == 1) {
                    cmsghdr *c = CMSG_FIRSTHDR(&msg);
                    if (status == 0 && c && c->cmsg_level == SOL_SOCKET && c->cmsg_type == SCM_RIGHTS) {
                        int fd = -1;
                        std::memcpy(&fd, CMSG_DATA(c), sizeof(int));
                        ::close(sock);
                        return fd;
                    }
                    ::close(sock);
                    throw std::runtime_error("fd server refused index " + std::to_string(index));
                }
                last = "no reply";
            } else {
                last = "send failed";
            }
        } else {
            last = std::strerror(errno);
        }
        ::close(sock);
        if (std::chrono::steady_clock::now() > deadline)
            throw std::runtime_error("fd client: cannot reach '" + name + "': " + last);
        std::this_thread::sleep_for(std::chrono::milliseconds(10));
    }
}

} // namespace engram
