// Test driver for the descriptor exchange of a tensor-parallel group
// (host/src/fd_exchange.cpp): one process of a group, run as
//   fd_exchange_driver <group> <gen> <rank> <world> <timeout_ms>
// It passes a memory file holding "token <rank>" and the size 1000 + rank, reads every
// descriptor it receives back from offset 0, and prints one JSON line: whether the exchange
// succeeded, the message on failure, each peer's token and size, and the number of open
// descriptors before the exchange and after closing the received ones (equal: none leaked).
#include <dirent.h>
#include <sys/mman.h>
#include <unistd.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "fd_exchange.h"

namespace {

int open_fds() {
    int n = 0;
    if (DIR* d = opendir("/proc/self/fd")) {
        while (readdir(d)) ++n;
        closedir(d);
    }
    return n;
}

std::string json_escape(const std::string& s) {
    std::string o;
    for (char c : s) {
        if (c == '"' || c == '\\') o += '\\';
        o += c;
    }
    return o;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 6) return 2;
    const unsigned long long group = std::strtoull(argv[1], nullptr, 16);
    const int gen = std::atoi(argv[2]), rank = std::atoi(argv[3]), world = std::atoi(argv[4]);
    const int timeout_ms = std::atoi(argv[5]);
    const int fd = memfd_create("qwc-exchange-test", MFD_CLOEXEC);
    if (fd < 0) return 3;
    const std::string token = "token " + std::to_string(rank);
    if (pwrite(fd, token.data(), token.size(), 0) != (ssize_t)token.size()) return 3;
    const int before = open_fds();
    int fds[qwc::kFdExchangeMaxRanks];
    uint64_t sizes[qwc::kFdExchangeMaxRanks];
    std::string why;
    const bool ok = qwc::exchange_fds(group, gen, rank, world, fd, 1000 + rank, timeout_ms, fds, sizes, why);
    std::string peers;
    for (int q = 0; ok && q < world; ++q) {
        if (q == rank) continue;
        char buf[64] = {};
        const ssize_t n = pread(fds[q], buf, sizeof(buf) - 1, 0);
        if (!peers.empty()) peers += ", ";
        peers += "\"" + std::to_string(q) + "\": [\"" + json_escape(std::string(buf, n > 0 ? n : 0)) + "\", " +
                 std::to_string((unsigned long long)sizes[q]) + "]";
        close(fds[q]);
    }
    const int after = open_fds();
    std::printf("{\"ok\": %s, \"why\": \"%s\", \"peers\": {%s}, \"fds_before\": %d, \"fds_after\": %d}\n",
                ok ? "true" : "false", json_escape(why).c_str(), peers.c_str(), before, after);
    close(fd);
    return ok ? 0 : 1;
}
