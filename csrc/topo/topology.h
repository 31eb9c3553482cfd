// Platform discovery from sysfs (no libnuma dependency: NUMA placement and
// page-node queries use the mbind/move_pages system calls directly).
//
// Parity: reference src/mpcomm.cpp:2822-3369 (NUMA, NIC NUMA, GPU BDF ->
// NUMA, PCIe affinity by longest common sysfs path prefix, suffix
// extraction) and :98-138 (NUMA-local allocation).
#ifndef MPCOMM_B200_CSRC_TOPO_TOPOLOGY_H_
#define MPCOMM_B200_CSRC_TOPO_TOPOLOGY_H_

#include <cstddef>
#include <string>
#include <vector>

namespace mpcomm {
namespace topo {

// Root of sysfs; MPCOMM_SYSFS_ROOT overrides it (tests use a fake tree).
const std::string &sysfs_root();

// Number of NUMA nodes (>= 1).
int numa_node_count();
// CPUs of a NUMA node (parsed cpulist); empty if unknown.
std::vector<int> numa_cpus(int node);
// Parses a kernel cpulist such as "0-3,8,10-11".
std::vector<int> parse_cpulist(const std::string &s);
// NUMA node of a PCI device given its BDF ("0000:53:00.0"); -1 if unknown.
int pci_numa_node(const std::string &bdf);
// Canonical sysfs path of a PCI device; empty if unknown.
std::string pci_realpath(const std::string &bdf);
// NUMA node / sysfs path of an RDMA device (/sys/class/infiniband/<nic>).
int ib_numa_node(const std::string &nic);
std::string ib_realpath(const std::string &nic);
std::vector<std::string> ib_device_names();
// Length of the common prefix of two sysfs paths, counted in whole path
// components (so ".../pci0000:10/0000:10:01.0" vs ".../0000:10:01.1" do not
// share the last component).
size_t common_path_components(const std::string &a, const std::string &b);
// Indices of `paths` that share the longest common path with `target` (all
// of them tied at the maximum, and only if the maximum reaches below the
// root complex, i.e. > 3 components).
std::vector<size_t> best_affinity(const std::string &target, const std::vector<std::string> &paths);
// Trailing decimal number of a device name ("mlx5_3" -> 3, "nvl_12" -> 12,
// "eth" -> -1).
int name_suffix(const std::string &name);
// NUMA node of the page holding `addr` (move_pages query); -1 if unknown.
int numa_node_of_addr(const void *addr);
// mmap + mbind(MPOL_PREFERRED) + first touch; node < 0 = no policy.
void *numa_alloc(size_t bytes, int node);
void numa_free(void *p, size_t bytes);
// Pins the calling thread to `cpus` intersected with its current affinity.
bool bind_thread_to_cpus(const std::vector<int> &cpus);

// Host DRAM bandwidth seen by the CPUs, independent of any device: `threads`
// threads (0 = one per CPU of this process's affinity, each pinned to one)
// stream over disjoint slices of one `bytes` buffer on NUMA node `node`
// (-1 = no policy). Best of `reps` passes, GB/s (1e9): write = memset,
// read = 64-bit sums of every word. Returns false when allocation fails.
struct HostBandwidth {
    double write_gbs = 0;
    double read_gbs = 0;
    int threads = 0;
};
bool host_bandwidth(size_t bytes, int threads, int node, int reps, HostBandwidth *out);

}  // namespace topo
}  // namespace mpcomm

#endif  // MPCOMM_B200_CSRC_TOPO_TOPOLOGY_H_
