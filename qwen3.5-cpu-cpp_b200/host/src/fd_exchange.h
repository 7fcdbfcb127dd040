// Exchange of file descriptors between the processes of a group on one host, over abstract
// Unix sockets (no files, no network): used to share the peer-memory buffers of a
// tensor-parallel group (each rank's buffer is exported as a file descriptor).
#pragma once
#include <cstdint>
#include <string>

namespace qwc {

constexpr int kFdExchangeMaxRanks = 8;

// Collective over the `world` processes of a group: sends `fd` (with the size `bytes`) to
// every other rank and receives every other rank's descriptor and size. The sockets are
// named after (group, gen, rank), so the processes must share a network namespace; `gen`
// separates successive exchanges of one group. On success fds[q] / sizes[q] hold rank q's
// descriptor (a new descriptor of this process, owned by the caller) and size for every
// q != rank, and fds[rank] = -1. On failure (a rank that does not take part within
// timeout_ms, a malformed message) nothing is left open and `why` says what went wrong.
// `fd` stays open and owned by the caller either way.
bool exchange_fds(uint64_t group, int gen, int rank, int world, int fd, uint64_t bytes, int timeout_ms,
                  int* fds, uint64_t* sizes, std::string& why);

}  // namespace qwc
