// Symmetric peer-mapped workspace: allocation, CUDA IPC export / import, status word.
#include "workspace.h"

#include <c10/util/Exception.h>

#include <cstring>

namespace qfc {

namespace {
void cuda_check(cudaError_t e, const char* what) {
  TORCH_CHECK(e == cudaSuccess, "qfc workspace: ", what, " failed: ", cudaGetErrorString(e));
}

struct DeviceScope {
  int prev = -1;
  explicit DeviceScope(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cuda_check(cudaSetDevice(dev), "cudaSetDevice");
  }
  ~DeviceScope() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};
}  // namespace

Workspace::Workspace(int64_t device, int64_t rank, int64_t world, int64_t rs_bytes, int64_t ag_bytes,
                     int64_t os_bytes)
    : device_(device), rank_(rank), world_(world) {
  TORCH_CHECK(world >= 1 && world <= kMaxRanks, "qfc workspace: world size must be in [1, 8]");
  TORCH_CHECK(rank >= 0 && rank < world, "qfc workspace: bad rank");
  rs_bytes_ = align_up(std::max<int64_t>(rs_bytes, 256), 4096);
  ag_bytes_ = align_up(std::max<int64_t>(ag_bytes, 256), 4096);
  os_bytes_ = align_up(std::max<int64_t>(os_bytes, 256), 4096);
  total_bytes_ = kFlagBytes + kArgmaxBytes + rs_bytes_ + ag_bytes_ + 2 * os_bytes_;
  DeviceScope scope((int)device);
  cuda_check(cudaMalloc(&base_, total_bytes_), "cudaMalloc(workspace)");
  cuda_check(cudaMemset(base_, 0, kFlagBytes), "cudaMemset(flags)");
  cuda_check(cudaMalloc(&epochs_, sizeof(uint32_t) * kEpochAlgos * kMaxBlocks), "cudaMalloc(epochs)");
  cuda_check(cudaMemset(epochs_, 0, sizeof(uint32_t) * kEpochAlgos * kMaxBlocks), "cudaMemset(epochs)");
  void* h = nullptr;
  cuda_check(cudaHostAlloc(&h, sizeof(KernelStatus), cudaHostAllocMapped | cudaHostAllocPortable),
             "cudaHostAlloc(status)");
  status_host_ = reinterpret_cast<KernelStatus*>(h);
  std::memset(status_host_, 0, sizeof(KernelStatus));
  void* d = nullptr;
  cuda_check(cudaHostGetDevicePointer(&d, h, 0), "cudaHostGetDevicePointer(status)");
  status_dev_ = reinterpret_cast<KernelStatus*>(d);
  cuda_check(cudaDeviceSynchronize(), "cudaDeviceSynchronize(workspace init)");
  peers_.assign(world, nullptr);
  peer_opened_.assign(world, false);
  peers_[rank] = base_;
  peers_ready_ = (world == 1);
}

Workspace::~Workspace() {
  DeviceScope scope((int)device_);
  for (size_t r = 0; r < peers_.size(); ++r) {
    if (peer_opened_[r] && peers_[r] != nullptr) cudaIpcCloseMemHandle(peers_[r]);
  }
  if (base_) cudaFree(base_);
  if (epochs_) cudaFree(epochs_);
  if (status_host_) cudaFreeHost(status_host_);
}

std::string Workspace::ipc_handle() const {
  DeviceScope scope((int)device_);
  cudaIpcMemHandle_t h;
  cuda_check(cudaIpcGetMemHandle(&h, base_), "cudaIpcGetMemHandle");
  return std::string(reinterpret_cast<const char*>(&h), sizeof(h));
}

void Workspace::open_peers(const std::vector<std::string>& handles) {
  TORCH_CHECK((int64_t)handles.size() == world_, "open_peers: expected one handle per rank");
  DeviceScope scope((int)device_);
  for (int64_t r = 0; r < world_; ++r) {
    if (r == rank_) continue;
    TORCH_CHECK(handles[r].size() == sizeof(cudaIpcMemHandle_t), "open_peers: bad handle size");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handles[r].data(), sizeof(h));
    void* p = nullptr;
    cuda_check(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
    peers_[r] = reinterpret_cast<char*>(p);
    peer_opened_[r] = true;
  }
  peers_ready_ = true;
}

void Workspace::set_peer_ptrs(const std::vector<int64_t>& ptrs) {
  TORCH_CHECK((int64_t)ptrs.size() == world_, "set_peer_ptrs: expected one pointer per rank");
  for (int64_t r = 0; r < world_; ++r) {
    peers_[r] = reinterpret_cast<char*>(ptrs[r]);
    peer_opened_[r] = false;
  }
  peers_ready_ = true;
}

std::vector<int64_t> Workspace::status() const {
  volatile KernelStatus* s = status_host_;
  return {s->code, s->phase, s->block, s->peer, (int64_t)s->want, (int64_t)s->seen};
}

void Workspace::clear_status() { std::memset(status_host_, 0, sizeof(KernelStatus)); }

}  // namespace qfc
