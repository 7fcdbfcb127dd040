// Descriptor exchange of a process group over abstract Unix sockets (see fd_exchange.h).
//
// Every rank listens on its own socket, then connects to each other rank's socket (retrying
// until that rank listens) and sends one message {magic, rank, bytes} with its descriptor
// attached (SCM_RIGHTS), then accepts the other ranks' connections and receives theirs.
// A connection is queued by the listener's backlog until it is accepted, so the sends do
// not wait for the receivers and no rank can block another: every rank sends all, then
// receives all. Every wait is bounded by the caller's timeout.
#include "fd_exchange.h"

#include <poll.h>
#include <sys/socket.h>
#include <sys/time.h>
#include <sys/un.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <chrono>
#include <cstddef>
#include <cstdio>
#include <cstring>
#include <thread>

namespace qwc {

namespace {

constexpr uint32_t kMagic = 0x71776332u;

struct Msg {
    uint32_t magic, rank;
    uint64_t bytes;
};

double now_ms() {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

// abstract socket address of (group, generation, rank)
socklen_t sock_addr(sockaddr_un& a, uint64_t group, int gen, int rank) {
    std::memset(&a, 0, sizeof(a));
    a.sun_family = AF_UNIX;
    const int n = std::snprintf(a.sun_path + 1, sizeof(a.sun_path) - 1, "qwc-p2p-%016llx-%d-%d",
                                (unsigned long long)group, gen, rank);
    return (socklen_t)(offsetof(sockaddr_un, sun_path) + 1 + n);
}

bool send_fd(int sock, const Msg& m, int fd) {
    iovec iov{const_cast<Msg*>(&m), sizeof(m)};
    alignas(cmsghdr) char cbuf[CMSG_SPACE(sizeof(int))];
    std::memset(cbuf, 0, sizeof(cbuf));
    msghdr h{};
    h.msg_iov = &iov;
    h.msg_iovlen = 1;
    h.msg_control = cbuf;
    h.msg_controllen = sizeof(cbuf);
    cmsghdr* c = CMSG_FIRSTHDR(&h);
    c->cmsg_level = SOL_SOCKET;
    c->cmsg_type = SCM_RIGHTS;
    c->cmsg_len = CMSG_LEN(sizeof(int));
    std::memcpy(CMSG_DATA(c), &fd, sizeof(int));
    return sendmsg(sock, &h, MSG_NOSIGNAL) == (ssize_t)sizeof(m);
}

bool recv_fd(int sock, Msg& m, int& fd) {
    iovec iov{&m, sizeof(m)};
    alignas(cmsghdr) char cbuf[CMSG_SPACE(sizeof(int))];
    msghdr h{};
    h.msg_iov = &iov;
    h.msg_iovlen = 1;
    h.msg_control = cbuf;
    h.msg_controllen = sizeof(cbuf);
    const ssize_t n = recvmsg(sock, &h, 0);
    // a descriptor that arrived is taken (and closed by the caller on failure) even when
    // the message around it is short, so none stays open unnoticed
    cmsghdr* c = n > 0 ? CMSG_FIRSTHDR(&h) : nullptr;
    if (c && c->cmsg_level == SOL_SOCKET && c->cmsg_type == SCM_RIGHTS) std::memcpy(&fd, CMSG_DATA(c), sizeof(int));
    return n == (ssize_t)sizeof(m) && fd >= 0 && m.magic == kMagic;
}

}  // namespace

bool exchange_fds(uint64_t group, int gen, int rank, int world, int fd, uint64_t bytes, int timeout_ms,
                  int* fds, uint64_t* sizes, std::string& why) {
    if (world < 2 || world > kFdExchangeMaxRanks || rank < 0 || rank >= world || fd < 0) {
        why = "exchange: group size outside 2..8, bad rank or descriptor";
        return false;
    }
    for (int q = 0; q < world; ++q) {
        fds[q] = -1;
        sizes[q] = 0;
    }
    const int lsock = socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
    if (lsock < 0) {
        why = std::string("socket: ") + std::strerror(errno);
        return false;
    }
    sockaddr_un la;
    const socklen_t llen = sock_addr(la, group, gen, rank);
    if (bind(lsock, reinterpret_cast<sockaddr*>(&la), llen) != 0 || listen(lsock, kFdExchangeMaxRanks) != 0) {
        why = std::string("bind/listen: ") + std::strerror(errno);
        close(lsock);
        return false;
    }
    const double t0 = now_ms();
    bool ok = true;
    // ---- send ours to every other rank
    for (int q = 0; q < world && ok; ++q) {
        if (q == rank) continue;
        sockaddr_un pa;
        const socklen_t plen = sock_addr(pa, group, gen, q);
        for (;;) {
            const int s = socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
            if (s >= 0 && connect(s, reinterpret_cast<sockaddr*>(&pa), plen) == 0) {
                const Msg m{kMagic, (uint32_t)rank, bytes};
                ok = send_fd(s, m, fd);
                close(s);
                if (!ok) why = "sending the descriptor to rank " + std::to_string(q) + " failed";
                break;
            }
            if (s >= 0) close(s);
            if (now_ms() - t0 > timeout_ms) {
                ok = false;
                why = "rank " + std::to_string(q) + " did not open its exchange socket in time";
                break;
            }
            std::this_thread::sleep_for(std::chrono::milliseconds(2));
        }
    }
    // ---- receive every other rank's
    for (int got = 0; ok && got < world - 1;) {
        pollfd p{lsock, POLLIN, 0};
        const int left = (int)std::max(1.0, timeout_ms - (now_ms() - t0));
        if (poll(&p, 1, left) <= 0) {
            ok = false;
            why = "a rank's descriptor did not arrive in time";
            break;
        }
        const int s = accept4(lsock, nullptr, nullptr, SOCK_CLOEXEC);
        if (s < 0) continue;
        timeval tv{5, 0};
        setsockopt(s, SOL_SOCKET, SO_RCVTIMEO, &tv, sizeof(tv));
        Msg m{};
        int rfd = -1;
        if (recv_fd(s, m, rfd) && (int)m.rank < world && (int)m.rank != rank && fds[m.rank] < 0) {
            fds[m.rank] = rfd;
            sizes[m.rank] = m.bytes;
            ++got;
        } else if (rfd >= 0) {
            close(rfd);
        }
        close(s);
    }
    close(lsock);
    if (!ok) {
        for (int q = 0; q < world; ++q)
            if (fds[q] >= 0) {
                close(fds[q]);
                fds[q] = -1;
            }
    }
    return ok;
}

}  // namespace qwc
