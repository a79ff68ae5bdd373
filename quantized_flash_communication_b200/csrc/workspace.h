// Symmetric peer-mapped workspace for the fused cross-GPU kernels.
//
// Every rank of a communicator owns one device buffer of identical size and layout;
// CUDA IPC handles are exchanged once (the Python layer moves the 64-byte handles over
// torch.distributed) and every rank maps every peer's buffer, so a kernel can store
// straight into a peer's memory over NVLink / NVSwitch.
//
// Buffer layout (byte offsets, identical on every rank):
//   [0, kFlagBytes)                     flags[phase][block][src_rank]  (uint32)
//   [kFlagBytes, + kArgmaxBytes)        argmax gather slots, double-buffered by epoch parity
//   [rs_off, rs_off + rs_bytes)         two-shot reduce-scatter slots (one per source rank)
//   [ag_off, ag_off + ag_bytes)         two-shot all-gather slots      (one per source rank)
//   [os_off, os_off + 2 * os_bytes)     one-shot slots, double-buffered by the parity of the
//                                       rank's count of one-shot calls
// Per-block epoch counters and the host-mapped status word are local to the rank.
//
// The reference has no counterpart: it moves every byte through NCCL collectives
// (communication.py:48-50, 79-81).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

#include "status.h"

namespace qfc {

constexpr int kMaxRanks = 8;
constexpr int kMaxBlocks = 1024;
constexpr int kFlagPhases = 5;   // 0 reduce-scatter, 1 all-gather, 2 one-shot, 3 GEMM-fused scatter, 4 argmax
constexpr int kEpochAlgos = 5;   // per-algorithm epoch counters
constexpr int64_t kFlagBytes = (int64_t)kFlagPhases * kMaxBlocks * kMaxRanks * sizeof(uint32_t);
// Cross-rank argmax: up to kArgmaxRows (score, index) pairs of 8 bytes per source rank.
constexpr int64_t kArgmaxRows = 512;
constexpr int64_t kArgmaxBytes = 2 * kMaxRanks * kArgmaxRows * 8;

// The two-shot kernels' grids stay below this many CTAs; the staged two-shot kernel
// publishes its second stage's flags at block index b + kStageBlockOff.
constexpr int kStageBlockOff = kMaxBlocks / 2;

// Two words of the one-shot epoch row that are not block epochs (the one-shot grid stays
// below them): the rank's count of finished one-shot calls, whose parity selects the slot
// region of a call, and the number of CTAs of the running call that have finished.
constexpr int kOneShotCallsWord = kMaxBlocks - 1;
constexpr int kOneShotDoneWord = kMaxBlocks - 2;

enum FlagPhase : int { PH_RS = 0, PH_AG = 1, PH_OS = 2, PH_GEMM = 3, PH_ARGMAX = 4 };
enum EpochAlgo : int { ALG_TWO_SHOT = 0, ALG_ONE_SHOT = 1, ALG_GEMM_RS = 2, ALG_GEMM_AG = 3, ALG_ARGMAX = 4 };

inline int64_t align_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

class Workspace {
 public:
  // Allocates this rank's buffer.  rs_bytes / ag_bytes / os_bytes are the capacities of
  // the three slot regions (each holds world slots).
  Workspace(int64_t device, int64_t rank, int64_t world, int64_t rs_bytes, int64_t ag_bytes,
            int64_t os_bytes);
  ~Workspace();
  Workspace(const Workspace&) = delete;
  Workspace& operator=(const Workspace&) = delete;

  // 64-byte CUDA IPC handle of the local buffer.
  std::string ipc_handle() const;
  // Map every peer's buffer from its IPC handle (index = rank; own entry ignored).
  void open_peers(const std::vector<std::string>& handles);
  // Same-process peers (single-GPU emulation of several ranks): raw device pointers.
  void set_peer_ptrs(const std::vector<int64_t>& ptrs);

  int64_t local_ptr() const { return reinterpret_cast<int64_t>(base_); }
  int64_t device() const { return device_; }
  int64_t rank() const { return rank_; }
  int64_t world() const { return world_; }
  int64_t rs_bytes() const { return rs_bytes_; }
  int64_t ag_bytes() const { return ag_bytes_; }
  int64_t os_bytes() const { return os_bytes_; }
  int64_t argmax_off() const { return kFlagBytes; }
  int64_t rs_off() const { return kFlagBytes + kArgmaxBytes; }
  int64_t ag_off() const { return rs_off() + rs_bytes_; }
  int64_t os_off() const { return rs_off() + rs_bytes_ + ag_bytes_; }
  bool peers_ready() const { return peers_ready_; }

  char* base() const { return base_; }
  char* peer_base(int r) const { return peers_[r]; }
  uint32_t* epochs() const { return epochs_; }
  KernelStatus* status_dev() const { return status_dev_; }

  // (code, phase, block, peer, want, seen) read from host-mapped memory, no sync.
  std::vector<int64_t> status() const;
  void clear_status();

 private:
  int64_t device_, rank_, world_;
  int64_t rs_bytes_, ag_bytes_, os_bytes_, total_bytes_;
  char* base_ = nullptr;
  std::vector<char*> peers_;
  std::vector<bool> peer_opened_;  // true where the pointer came from cudaIpcOpenMemHandle
  bool peers_ready_ = false;
  uint32_t* epochs_ = nullptr;
  KernelStatus* status_host_ = nullptr;
  KernelStatus* status_dev_ = nullptr;
};

}  // namespace qfc
