// NUMA placement of the pinned host tier.
//
// The reference assigns every manager the NUMA node of its device's PCI
// root (RaidenManagerBase::DetectAndAssignNumaNode,
// tpu_sync/core/raiden_manager_base.cc:47-78), or a caller-given override
// (KVCacheManagerBase ctor, tpu_sync/kv_cache/kv_cache_manager_base.cc:
// 231-249), and runs its DMA dispatch threads on that node.  Here the node
// decides where the host tier's pages live: while the tier is allocated and
// pinned, the allocating thread's memory policy prefers that node, so the
// pages sit next to the GPU's root port on a multi-socket host.  On a host
// with one NUMA node nothing is changed.  A kernel that refuses the policy
// call (a container without the permission) leaves the placement to the
// kernel's default; the manager reports whether it was applied.

#include <dirent.h>
#include <sys/syscall.h>
#include <unistd.h>

#include <cctype>
#include <cstdio>
#include <cstring>
#include <string>

#include <cuda_runtime.h>

#include "ts_internal.h"

namespace tsb {
namespace {

constexpr int kMpolDefault = 0;
constexpr int kMpolPreferred = 1;

std::string sysfs(const char* root) { return root && root[0] ? root : "/sys"; }

}  // namespace

int pci_numa_node(const char* bus_id, const char* sysfs_root) {
  if (!bus_id || !bus_id[0]) return -1;
  std::string id(bus_id);
  for (char& c : id) c = char(std::tolower(static_cast<unsigned char>(c)));
  // "00000000:1b:00.0" (CUDA's 8-digit domain) and "0000:1b:00.0" (sysfs)
  const size_t colon = id.find(':');
  if (colon != std::string::npos && colon > 4) id = id.substr(colon - 4);
  const std::string path = sysfs(sysfs_root) + "/bus/pci/devices/" + id + "/numa_node";
  FILE* f = std::fopen(path.c_str(), "r");
  if (!f) return -1;
  int node = -1;
  if (std::fscanf(f, "%d", &node) != 1) node = -1;
  std::fclose(f);
  return node < 0 ? -1 : node;
}

int numa_node_count(const char* sysfs_root) {
  const std::string dir = sysfs(sysfs_root) + "/devices/system/node";
  DIR* d = opendir(dir.c_str());
  if (!d) return 1;
  int n = 0;
  while (dirent* e = readdir(d)) {
    const char* s = e->d_name;
    if (std::strncmp(s, "node", 4) == 0 && std::isdigit(static_cast<unsigned char>(s[4]))) ++n;
  }
  closedir(d);
  return n > 0 ? n : 1;
}

int device_numa_node(int device) {
  char bus[32] = {0};
  if (cudaDeviceGetPCIBusId(bus, int(sizeof(bus)), device) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  return pci_numa_node(bus, nullptr);
}

ScopedPreferredNode::ScopedPreferredNode(int node) {
  if (node < 0 || node >= kMaskWords * 64) return;
  // the thread's policy before, restored on exit
  if (syscall(SYS_get_mempolicy, &prev_mode_, prev_mask_, kMaskWords * 64 + 1, nullptr, 0) != 0)
    prev_mode_ = kMpolDefault;
  unsigned long mask[kMaskWords] = {0};
  mask[node / 64] = 1ul << (node % 64);
  applied_ = syscall(SYS_set_mempolicy, kMpolPreferred, mask, kMaskWords * 64 + 1) == 0;
}

ScopedPreferredNode::~ScopedPreferredNode() {
  if (!applied_) return;
  if (prev_mode_ == kMpolDefault ||
      syscall(SYS_set_mempolicy, prev_mode_, prev_mask_, kMaskWords * 64 + 1) != 0)
    syscall(SYS_set_mempolicy, kMpolDefault, nullptr, 0);
}

}  // namespace tsb

extern "C" int ts_pci_numa_node(const char* bus_id, const char* sysfs_root, int* node_out) {
  tsb::clear_error();
  if (!bus_id || !node_out) return tsb::set_error(TS_INVALID_ARGUMENT, "null pointer argument");
  *node_out = tsb::pci_numa_node(bus_id, sysfs_root);
  return TS_OK;
}
