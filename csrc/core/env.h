// Environment knobs and host-side fault injection.
//
// Knobs (all optional):
//   BCCL_LOG_LEVEL, BCCL_ALGO=oneshot|twoshot|nvls|ring, BCCL_DISABLE_NVLS=1,
//   BCCL_MAX_CTAS=<n>, BCCL_TIMEOUT_MS=<ms>, BCCL_BUFFSIZE=<bytes per peer slot>,
//   BCCL_TUNING_FILE=<path>, BCCL_BOOTSTRAP_TIMEOUT_MS=<ms>, BCCL_DISABLE_SHM=1,
//   BCCL_HOST_EXECUTOR=threads|polling|epoll.
// Parity: the reference's OCCL_* environment switches (OriginCCL src/communicator.cpp:47-60).
//
// Fault injection (BCCL_FAULT) exists for host-side failure tests only; nothing here can make
// a GPU fault or hang. Format: comma-separated "site:rank[:arg]" entries, e.g.
//   BCCL_FAULT=bootstrap_skip:2            rank 2 never joins the bootstrap
//   BCCL_FAULT=bootstrap_delay:1:500       rank 1 joins 500 ms late
//   BCCL_FAULT=bootstrap_corrupt:3         rank 3 sends a malformed hello
//   BCCL_FAULT=handle_drop:1               rank 1 never sends its memory handle fds
//   BCCL_FAULT=segment_drop:0              local leader 0 never shares the host segment
#pragma once

#include <cstdint>
#include <string>

namespace bccl {

long EnvInt(const char* name, long dflt);
std::string EnvStr(const char* name, const std::string& dflt);
bool EnvFlag(const char* name);  // "1", "true", "yes", "on"
// True when BCCL_FAULT lists `site` for `rank`; *arg receives the optional argument.
bool FaultActive(const char* site, int rank, long* arg = nullptr);

}  // namespace bccl
