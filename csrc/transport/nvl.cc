// "nvl" backend: B200 GPU fabric rails.
//
// One rail per visible GPU. A queue pair is a CUDA stream of that GPU; a
// posted WR is resolved to a (src, dst) device-address pair and queued; the
// doorbell (flush) turns every queued WR into one descriptor of a single
// copy_batch launch — the sm_100a bulk-copy kernel — followed by an event.
// The last CTA of every launch stores the launch's sequence number into a
// host-mapped completion word of its QP; poll() reads that word (no driver
// call on the hot path, so polling never contends for the CUDA driver's
// locks with other launches) and emits one completion per WR, so the
// engine sees RC-verbs semantics. An event per launch remains for error
// detection: it is queried only for a launch pending longer than a while.
//
// Reachable memory:
//   * this process's device memory on any GPU (peer access enabled),
//   * this process's host memory (pinned + mapped at registration; UVA),
//   * another process's device memory on the same host: registrations are
//     published in /dev/shm/mpcomm-nvl.<boot>.<pid> (key, range, CUDA IPC
//     handle) and opened with cudaIpcOpenMemHandle on first use; VMM
//     (cuMemCreate) memory, which CUDA IPC cannot export (NVLS group copies,
//     GPUDirect buffers, PyTorch expandable segments), is offered instead as
//     the POSIX handles of its allocations on the owner's descriptor server
//     (abstract Unix socket mpcomm-fd.<boot>.<pid>) and imported + mapped
//     back to back by the peer on first use,
//   * another process's host memory when it is a shared file mapping
//     (/dev/shm, hugetlbfs, any MAP_SHARED file): the record carries the
//     file path and offset; the peer maps the same pages, pins them and
//     reaches them through its own UVA address. Private anonymous memory of
//     another process is unreachable (WC remote-access error).
// This replaces the reference's NVLink proxy copies (cuMemcpyPeerAsync +
// host callbacks, src/mpcomm_pxn.cpp:638-814) with in-kernel stores.
#include <fcntl.h>
#include <signal.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <atomic>
#include <cerrno>
#include <chrono>
#include <cstring>
#include <deque>
#include <map>
#include <set>
#include <mutex>
#include <tuple>
#include <unordered_map>
#include <vector>

#include "core/core.h"
#include "core/nvtx.h"
#include "cuda/gpu.h"
#include "kernels/launch.h"
#include "mpcomm.h"
#include "mpcomm_log.h"
#include "parallel/vmm.h"
#include "topo/topology.h"
#include "transport/fabric.h"

namespace mpcomm {
namespace fabric {
namespace {

constexpr uint32_t kDirMagic = 0x4E564C4D;  // "NVLM": layout with file-backed host and multicast records
constexpr size_t kDirSlots = 4096;

struct DirRecord {
    uint32_t key;
    uint32_t state;  // 0 free, 1 valid, 2 being written
    uint64_t addr;
    uint64_t len;
    uint64_t base;
    uint64_t alloc_size;
    int32_t device;
    int32_t kind;  // 0 device memory (CUDA IPC), 1 host memory, 2 device memory (VMM, descriptor server)
    unsigned char ipc[gpu::kIpcHandleBytes];
    uint64_t file_off;  // host memory: offset of `addr` in the backing file
    char path[160];     // host memory: backing file ("" = private, unreachable)
    // NVLS group this registration is the owner's copy of (0 = none): `addr`
    // is the group buffer's offset 0 on the owner's GPU.
    uint32_t mc_members;
    uint32_t mc_pad;
    uint64_t mc_token;
};

// Backing file of a host range that lies inside one shared file mapping of
// this process (from /proc/self/maps): path and the file offset of `addr`.
bool shared_backing(uintptr_t addr, size_t len, std::string *path, uint64_t *off) {
    FILE *f = fopen("/proc/self/maps", "r");
    if (!f) return false;
    char line[512];
    bool found = false;
    while (fgets(line, sizeof(line), f)) {
        unsigned long lo = 0, hi = 0, foff = 0;
        char perms[8] = {0};
        int pos = 0;
        if (sscanf(line, "%lx-%lx %7s %lx %*s %*s %n", &lo, &hi, perms, &foff, &pos) < 4) continue;
        if (addr < lo || addr >= hi) continue;
        if (addr + len > hi || perms[3] != 's' || pos <= 0) break;
        std::string p(line + pos);
        while (!p.empty() && (p.back() == '\n' || p.back() == ' ')) p.pop_back();
        // Only a path another process can open (not "/memfd:... (deleted)").
        if (p.empty() || p[0] != '/' || p.find(" (deleted)") != std::string::npos) break;
        *path = p;
        *off = foff + (addr - lo);
        found = true;
        break;
    }
    fclose(f);
    return found;
}

struct DirHeader {
    uint32_t magic;
    uint32_t slots;
    uint64_t pid;
};

std::string boot_tag() {
    static const std::string tag = [] {
        char buf[64] = {0};
        FILE *f = fopen("/proc/sys/kernel/random/boot_id", "r");
        if (f) {
            if (!fgets(buf, sizeof(buf), f)) buf[0] = 0;
            fclose(f);
        }
        std::string s;
        for (char c : std::string(buf))
            if (std::isxdigit(static_cast<unsigned char>(c))) s.push_back(c);
        return s.substr(0, 8).empty() ? std::string("00000000") : s.substr(0, 8);
    }();
    return tag;
}

std::string dir_path(long pid) {
    return "/dev/shm/mpcomm-nvl." + boot_tag() + "." + std::to_string(pid);
}

struct Region {
    uint32_t key;
    uintptr_t addr;
    size_t len;
    bool device;
    int dev;
    uintptr_t base;
    size_t alloc_size;
    bool pinned_by_us;
    int refs;
    size_t slot;
    std::string path;   // host memory: shared backing file ("" if private)
    uint64_t file_off;
    uint64_t mc_token = 0;    // NVLS group of which [addr, addr+len) is this process's copy
    uintptr_t mc_addr = 0;    // this process's multicast mapping of the group's offset 0
    int mc_members = 0;
    bool vmm = false;         // device memory offered as a VMM handle (kind 2)
};

// Multicast identity of a registration, as seen by a process posting to it.
struct McInfo {
    uint64_t token = 0;
    int members = 0;
    uintptr_t base = 0;  // owner's address of the group buffer's offset 0
};

// Process-wide registry of nvl registrations + the shared directory.
class Registry {
 public:
    static Registry &get() {
        static Registry r;
        return r;
    }

    int add(void *addr, size_t len, uint32_t *key) {
        std::lock_guard<std::mutex> g(mu_);
        for (auto &kv : regions_) {
            Region &r = kv.second;
            if (r.addr == reinterpret_cast<uintptr_t>(addr) && r.len == len) {
                ++r.refs;
                *key = r.key;
                return 0;
            }
        }
        Region r{};
        r.addr = reinterpret_cast<uintptr_t>(addr);
        r.len = len;
        gpu::PtrInfo info;
        bool known = gpu::query_pointer(addr, &info);
        unsigned char ipc[gpu::kIpcHandleBytes] = {0};
        if (known && info.is_device) {
            r.device = true;
            r.dev = info.device;
            r.base = info.base ? info.base : r.addr;
            r.alloc_size = info.size ? info.size : len;
            if (gpu::ipc_get_handle(reinterpret_cast<void *>(r.base), ipc) != 0) {
                // Not a cudaMalloc allocation: offer it as a VMM handle, else
                // it stays usable in-process only.
                std::memset(ipc, 0, sizeof(ipc));
                uintptr_t vb = 0;
                size_t span = 0;
                if (vmm::vmm_offer(addr, len, next_key_, &vb, &span) == 0) {
                    r.vmm = true;  // offered under the key assigned below
                    r.base = vb;
                    r.alloc_size = span;
                } else {
                    MPCOMM_LOG_DEBUG("MPComm[nvl]: device range %p+%zu is not exportable; other processes "
                                     "will not reach it\n", addr, len);
                }
            }
        } else {
            void *dptr = nullptr;
            bool pinned = false;
            int e = gpu::host_pin_mapped(addr, len, &dptr, &pinned);
            if (e != 0) {
                MPCOMM_LOG_ERROR("MPComm[nvl]: cannot pin host range %p+%zu: %s\n", addr, len,
                                 gpu::error_string(e));
                return MPCOMM_ERR_MEMORY;
            }
            if (dptr != addr) {
                // Non-UVA mapping: the kernels would need a translated pointer.
                if (pinned) gpu::host_unpin(addr);
                MPCOMM_LOG_ERROR("MPComm[nvl]: host memory %p is not identity-mapped\n", addr);
                return MPCOMM_ERR_MEMORY;
            }
            r.device = false;
            r.dev = -1;
            r.base = r.addr;
            r.alloc_size = len;
            r.pinned_by_us = pinned;
            if (!shared_backing(r.addr, len, &r.path, &r.file_off)) r.path.clear();
        }
        r.key = next_key_++;
        r.refs = 1;
        r.slot = publish(r, ipc);
        regions_[r.key] = r;
        *key = r.key;
        return 0;
    }

    int remove(uint32_t key) {
        std::lock_guard<std::mutex> g(mu_);
        auto it = regions_.find(key);
        if (it == regions_.end()) return MPCOMM_ERR_INVALID_ARG;
        if (--it->second.refs > 0) return 0;
        if (it->second.pinned_by_us) gpu::host_unpin(reinterpret_cast<void *>(it->second.addr));
        if (it->second.vmm) vmm::vmm_withdraw(key);
        if (dir_ && it->second.slot < kDirSlots) {
            DirRecord *rec = records() + it->second.slot;
            __atomic_store_n(&rec->state, 0u, __ATOMIC_RELEASE);
        }
        regions_.erase(it);
        return 0;
    }

    bool lookup(uint32_t key, Region *out) {
        std::lock_guard<std::mutex> g(mu_);
        auto it = regions_.find(key);
        if (it == regions_.end()) return false;
        *out = it->second;
        return true;
    }

    int set_multicast(uint32_t key, uintptr_t uc, size_t len, uintptr_t mc, uint64_t token, int members) {
        std::lock_guard<std::mutex> g(mu_);
        auto it = regions_.find(key);
        if (it == regions_.end() || !it->second.device || it->second.addr != uc || len > it->second.len ||
            !mc || !token || members < 2)
            return MPCOMM_ERR_INVALID_ARG;
        Region &r = it->second;
        r.mc_token = token;
        r.mc_addr = mc;
        r.mc_members = members;
        if (dir_ && r.slot < kDirSlots) {
            // Members before the token: a reader that sees the token sees a
            // member count too (or none, and then does not use multicast).
            DirRecord *rec = records() + r.slot;
            __atomic_store_n(&rec->mc_members, static_cast<uint32_t>(members), __ATOMIC_RELEASE);
            __atomic_store_n(&rec->mc_token, token, __ATOMIC_RELEASE);
        }
        return 0;
    }

    // This process's registration of NVLS group `token` (false if none).
    bool find_multicast(uint64_t token, Region *out) {
        std::lock_guard<std::mutex> g(mu_);
        for (auto &kv : regions_)
            if (kv.second.mc_token == token) {
                *out = kv.second;
                return true;
            }
        return false;
    }

    ~Registry() {
        if (dir_) {
            munmap(dir_, dir_bytes());
            unlink(dir_path(getpid()).c_str());
        }
    }

 private:
    static size_t dir_bytes() { return sizeof(DirHeader) + kDirSlots * sizeof(DirRecord); }
    DirRecord *records() {
        return reinterpret_cast<DirRecord *>(static_cast<char *>(dir_) + sizeof(DirHeader));
    }

    size_t publish(const Region &r, const unsigned char *ipc) {
        if (!dir_ && !dir_failed_) {
            std::string p = dir_path(getpid());
            int fd = open(p.c_str(), O_RDWR | O_CREAT | O_TRUNC, 0600);
            if (fd >= 0 && ftruncate(fd, static_cast<off_t>(dir_bytes())) == 0) {
                void *m = mmap(nullptr, dir_bytes(), PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
                if (m != MAP_FAILED) {
                    dir_ = m;
                    auto *h = static_cast<DirHeader *>(dir_);
                    h->slots = kDirSlots;
                    h->pid = static_cast<uint64_t>(getpid());
                    __atomic_store_n(&h->magic, kDirMagic, __ATOMIC_RELEASE);
                }
            }
            if (fd >= 0) close(fd);
            if (!dir_) {
                dir_failed_ = true;
                MPCOMM_LOG_WARN("MPComm[nvl]: cannot create %s; remote processes will not reach "
                                "this process's memory\n", p.c_str());
            }
        }
        if (!dir_) return kDirSlots;
        DirRecord *recs = records();
        for (size_t i = 0; i < kDirSlots; ++i) {
            if (__atomic_load_n(&recs[i].state, __ATOMIC_ACQUIRE) != 0) continue;
            __atomic_store_n(&recs[i].state, 2u, __ATOMIC_RELAXED);
            recs[i].key = r.key;
            recs[i].addr = r.addr;
            recs[i].len = r.len;
            recs[i].base = r.base;
            recs[i].alloc_size = r.alloc_size;
            recs[i].device = r.dev;
            recs[i].kind = !r.device ? 1 : r.vmm ? 2 : 0;
            std::memcpy(recs[i].ipc, ipc, gpu::kIpcHandleBytes);
            recs[i].file_off = r.file_off;
            std::memset(recs[i].path, 0, sizeof(recs[i].path));
            if (r.path.size() < sizeof(recs[i].path)) std::memcpy(recs[i].path, r.path.data(), r.path.size());
            recs[i].mc_members = 0;
            recs[i].mc_pad = 0;
            recs[i].mc_token = 0;
            __atomic_store_n(&recs[i].state, 1u, __ATOMIC_RELEASE);
            return i;
        }
        MPCOMM_LOG_WARN("MPComm[nvl]: registration directory full\n");
        return kDirSlots;
    }

    std::mutex mu_;
    std::map<uint32_t, Region> regions_;
    uint32_t next_key_ = 0x10000;
    void *dir_ = nullptr;
    bool dir_failed_ = false;
};

// Cache of other processes' directories and opened IPC mappings.
class RemoteMaps {
 public:
    static RemoteMaps &get() {
        static RemoteMaps m;
        return m;
    }
    // Resolves [addr, addr+len) of process `pid`'s registration `key` to a
    // pointer usable by kernels of this process on device `dev`. 0 on
    // success. Sets *host when the memory is host DRAM (a PCIe-bound copy).
    // IPC mappings belong to the context current when they are opened, so
    // they are opened with `dev` current and cached per (pid, base, dev).
    int resolve(long pid, uint32_t key, uintptr_t addr, size_t len, int dev, uintptr_t *out, bool *host,
                McInfo *mc = nullptr) {
        *host = false;
        std::lock_guard<std::mutex> g(mu_);
        DirRecord rec;
        const int found = find_record(pid, key, addr, len, &rec);
        if (found != 0) return found;
        if (mc) {
            mc->token = rec.mc_token;
            mc->members = static_cast<int>(rec.mc_members);
            mc->base = rec.addr;
        }
        const int prev = gpu::current_device();
        if (prev != dev) gpu::set_device(dev);
        int st;
        if (rec.kind == 1) {
            *host = true;
            st = resolve_host(pid, rec, addr, out);
        } else {
            st = resolve_device(pid, rec, addr, dev, out);
        }
        if (prev >= 0 && prev != dev) gpu::set_device(prev);
        return st;
    }
    // Multicast identity of process `pid`'s registration `key`, after the
    // same range check as resolve(), without mapping anything.
    int describe(long pid, uint32_t key, uintptr_t addr, size_t len, McInfo *mc) {
        std::lock_guard<std::mutex> g(mu_);
        DirRecord rec;
        const int found = find_record(pid, key, addr, len, &rec);
        if (found != 0) return found;
        mc->token = rec.mc_token;
        mc->members = static_cast<int>(rec.mc_members);
        mc->base = rec.addr;
        return 0;
    }

 private:
    // Copy of the live record `key` of `pid` covering [addr, addr+len).
    // Caller holds mu_.
    int find_record(long pid, uint32_t key, uintptr_t addr, size_t len, DirRecord *out) {
        const DirRecord *dir = open_dir(pid);
        if (!dir) return kWcRemAccessErr;
        for (size_t i = 0; i < kDirSlots; ++i) {
            if (__atomic_load_n(&dir[i].state, __ATOMIC_ACQUIRE) != 1 || dir[i].key != key) continue;
            DirRecord rec;
            std::memcpy(&rec, &dir[i], sizeof(rec));
            // The owner may free and reuse the slot while it is copied; keys
            // are never reused, so a slot still valid under the same key after
            // the copy held this record throughout.
            if (__atomic_load_n(&dir[i].state, __ATOMIC_ACQUIRE) != 1 ||
                __atomic_load_n(&dir[i].key, __ATOMIC_RELAXED) != key || rec.key != key)
                continue;
            if (addr < rec.addr || addr + len > rec.addr + rec.len) return kWcRemAccessErr;
            *out = rec;
            return 0;
        }
        return kWcRemAccessErr;
    }

    const DirRecord *open_dir(long pid) {
        auto it = dirs_.find(pid);
        if (it != dirs_.end()) return it->second;
        int fd = open(dir_path(pid).c_str(), O_RDONLY);
        if (fd < 0) return nullptr;
        size_t bytes = sizeof(DirHeader) + kDirSlots * sizeof(DirRecord);
        void *m = mmap(nullptr, bytes, PROT_READ, MAP_SHARED, fd, 0);
        close(fd);
        if (m == MAP_FAILED) return nullptr;
        auto *h = static_cast<const DirHeader *>(m);
        if (__atomic_load_n(&h->magic, __ATOMIC_ACQUIRE) != kDirMagic) {
            munmap(m, bytes);
            return nullptr;
        }
        const DirRecord *recs =
            reinterpret_cast<const DirRecord *>(static_cast<const char *>(m) + sizeof(DirHeader));
        dirs_[pid] = recs;
        return recs;
    }

 public:
    // Another process's shared host mapping: map the same file range here,
    // pin it (mapped, portable) and cache the local base per (pid, key).
    int resolve_host(long pid, const DirRecord &rec, uintptr_t addr, uintptr_t *out) {
        auto mk = std::make_pair(pid, rec.key);
        auto it = host_ranges_.find(mk);
        if (it == host_ranges_.end()) {
            if (rec.path[0] != '/') {
                MPCOMM_LOG_WARN("MPComm[nvl]: pid %ld's host buffer 0x%lx is private memory; publish a "
                                "shared mapping (e.g. /dev/shm) to reach it from another process\n",
                                pid, static_cast<unsigned long>(rec.addr));
                return kWcRemAccessErr;
            }
            std::string path(rec.path, strnlen(rec.path, sizeof(rec.path)));
            const uint64_t page = static_cast<uint64_t>(sysconf(_SC_PAGESIZE));
            const uint64_t off0 = rec.file_off & ~(page - 1);
            const size_t span = static_cast<size_t>(rec.file_off - off0 + rec.len);
            int fd = open(path.c_str(), O_RDWR);
            if (fd < 0) return kWcRemAccessErr;
            void *m = mmap(nullptr, span, PROT_READ | PROT_WRITE, MAP_SHARED, fd, static_cast<off_t>(off0));
            close(fd);
            if (m == MAP_FAILED) return kWcRemAccessErr;
            char *base = static_cast<char *>(m) + (rec.file_off - off0);
            void *dptr = nullptr;
            bool pinned = false;
            if (gpu::host_pin_mapped(base, rec.len, &dptr, &pinned) != 0 || dptr != base) {
                if (pinned) gpu::host_unpin(base);
                munmap(m, span);
                MPCOMM_LOG_ERROR("MPComm[nvl]: cannot pin %s (pid %ld) for device access\n", path.c_str(), pid);
                return kWcRemAccessErr;
            }
            it = host_ranges_.emplace(mk, reinterpret_cast<uintptr_t>(base)).first;
        }
        *out = it->second + (addr - rec.addr);
        return 0;
    }

    // VMM memory of `pid`: fetch the handles of the allocations behind the
    // registration from the owner's descriptor server and map them back to
    // back for `dev`, once per (pid, key, dev) (keys are never reused, so a
    // re-registered range is mapped afresh).
    int resolve_vmm(long pid, const DirRecord &rec, uintptr_t addr, int dev, uintptr_t *out) {
        auto mk = std::make_tuple(pid, rec.key, dev);
        auto it = vmm_opened_.find(mk);
        if (it == vmm_opened_.end()) {
            void *p = nullptr;
            std::vector<size_t> sizes;
            int e = vmm::vmm_open(pid, rec.key, dev, 5000, &p, &sizes);
            size_t span = 0;
            for (size_t n : sizes) span += n;
            if (e == 0 && span != rec.alloc_size) {
                vmm::vmm_unmap(p, sizes);
                e = -2;
            }
            if (e != 0) {
                MPCOMM_LOG_ERROR("MPComm[nvl]: pid %ld's VMM buffer 0x%lx: %s (%d)\n", pid,
                                 static_cast<unsigned long>(rec.addr),
                                 e == vmm::kVmmNotOffered ? "withdrawn"
                                 : e == vmm::kVmmUnreachable ? "owner unreachable"
                                                             : "cannot map",
                                 e);
                return kWcRemAccessErr;
            }
            it = vmm_opened_.emplace(mk, reinterpret_cast<uintptr_t>(p)).first;
        }
        *out = it->second + (addr - rec.base);
        return 0;
    }

    int resolve_device(long pid, const DirRecord &rec, uintptr_t addr, int dev, uintptr_t *out) {
        if (rec.kind == 2) return resolve_vmm(pid, rec, addr, dev, out);
        auto mk = std::make_tuple(pid, rec.base, dev);
        auto it = opened_.find(mk);
        if (it == opened_.end()) {
            bool any = false;
            for (size_t b = 0; b < gpu::kIpcHandleBytes; ++b) any |= rec.ipc[b] != 0;
            if (!any) return kWcRemAccessErr;
            void *p = nullptr;
            int e = gpu::ipc_open_handle(rec.ipc, &p);
            if (e != 0) {
                MPCOMM_LOG_ERROR("MPComm[nvl]: cudaIpcOpenMemHandle(pid %ld) failed: %s\n", pid,
                                 gpu::error_string(e));
                return kWcRemAccessErr;
            }
            it = opened_.emplace(mk, reinterpret_cast<uintptr_t>(p)).first;
        }
        *out = it->second + (addr - rec.base);
        return 0;
    }

    std::mutex mu_;
    std::unordered_map<long, const DirRecord *> dirs_;
    std::map<std::tuple<long, uintptr_t, int>, uintptr_t> opened_;  // (pid, base, local dev)
    std::map<std::tuple<long, uint32_t, int>, uintptr_t> vmm_opened_;  // (pid, key, local dev)
    std::map<std::pair<long, uint32_t>, uintptr_t> host_ranges_;  // portable pinned: any device
};

// gid = "nvl:<boot8>:<pid>:<dev>"
bool parse_gid(const std::string &gid, std::string *boot, long *pid, int *dev) {
    if (gid.compare(0, 4, "nvl:") != 0) return false;
    size_t a = gid.find(':', 4);
    if (a == std::string::npos) return false;
    size_t b = gid.find(':', a + 1);
    if (b == std::string::npos) return false;
    *boot = gid.substr(4, a - 4);
    *pid = std::strtol(gid.c_str() + a + 1, nullptr, 10);
    *dev = static_cast<int>(std::strtol(gid.c_str() + b + 1, nullptr, 10));
    return true;
}

class NvlRail;

struct Inflight {
    void *event;
    uint64_t seq;  // value the launch's last CTA stores into the QP's done word
    std::vector<uint64_t> wr_ids;
    std::vector<uint32_t> lens;
    std::chrono::steady_clock::time_point launched;
    bool failed;
};

// A launch not retired through its done word after this long is checked
// through its event (errors, lost context); later checks are spaced as much.
constexpr auto kEventCheckAfter = std::chrono::microseconds(500);

class NvlQp final : public QueuePair {
 public:
    NvlQp(NvlRail *rail, uint32_t qpn);
    ~NvlQp() override;
    uint32_t qp_num() const override { return qpn_; }
    QpState state() const override { return state_.load(); }
    int to_init() override {
        state_ = QpState::kInit;
        return 0;
    }
    int to_rtr(const EndpointInfo &remote) override;
    int to_rts() override {
        if (state_.load() != QpState::kRtr) return MPCOMM_ERR_CONNECTION;
        state_ = QpState::kRts;
        return 0;
    }
    int to_err() override;
    int recover() override {
        to_err();
        state_ = QpState::kInit;
        EndpointInfo r = remote_;
        if (to_rtr(r) != 0) return MPCOMM_ERR_CONNECTION;
        return to_rts();
    }
    int post(const WorkRequest *wrs, size_t n) override;
    int post_fanout(const WorkRequest &wr, const FanoutTarget *targets, size_t n, void *h2d_window) override;
    int post_paged(const PagedWrite &w) override;
    void flush() override;
    // Retires completed launches into the rail CQ. Caller holds rail mutex.
    void reap(std::deque<WorkCompletion> *cq);

 private:
    friend class NvlRail;
    NvlRail *rail_;
    uint32_t qpn_;
    std::atomic<QpState> state_{QpState::kReset};
    EndpointInfo remote_;
    long remote_pid_ = -1;
    int remote_dev_ = -1;
    void *stream_ = nullptr;
    uint32_t *status_ = nullptr;     // device: [0] status word, [4] last-CTA counter
    uint64_t *done_word_ = nullptr;  // host-mapped: sequence of the last finished launch
    uint64_t seq_ = 0;
    std::chrono::steady_clock::time_point next_check_{};
    std::vector<kern::CopyDesc> pending_;
    std::vector<uint64_t> pending_ids_;
    std::vector<uint32_t> pending_lens_;
    bool pending_host_ = false;
    bool pending_h2d_ = false;  // a READ from host memory into this GPU's HBM
    // One-to-many WRITEs queued since the last flush: one launch each.
    struct PendingFanout {
        const void *src;
        std::vector<void *> dsts;  // P2P sink (empty with a multicast sink)
        void *mc;                  // multicast address of the common offset (NVLS sink)
        uint32_t bytes;
        uint64_t wr_id;
        kern::H2DWindow *win;      // QoS window of a host-memory source (may be null)
    };
    std::vector<PendingFanout> pending_fanout_;
    // Paged WRITEs queued since the last flush: one pxn_gather_forward each.
    struct PendingPaged {
        PagedWrite w;
        void *dst;
    };
    std::vector<PendingPaged> pending_paged_;
    // Resolves a remote range of this QP's peer to a device pointer on this
    // rail's GPU (kWcSuccess or a WC error status); fills *mc if non-null.
    int resolve_remote(uint32_t rkey, uintptr_t raddr, size_t len, uintptr_t *out, bool *host, McInfo *mc);
    // Multicast identity of a remote range of this QP's peer (no mapping).
    int describe_remote(uint32_t rkey, uintptr_t raddr, size_t len, McInfo *mc);
    std::deque<Inflight> inflight_;
};

class NvlRail final : public Rail {
 public:
    NvlRail(int dev, const Config &cfg) : dev_(dev), cfg_(cfg) {
        name_ = "nvl_" + std::to_string(dev);
        gid_ = "nvl:" + boot_tag() + ":" + std::to_string(getpid()) + ":" + std::to_string(dev);
        std::string bdf = gpu::pci_bdf(dev);
        numa_ = topo::pci_numa_node(bdf);
        if (numa_ < 0) numa_ = 0;
        pci_path_ = topo::pci_realpath(bdf);
        sms_ = kern::sm_count(dev);
        std::lock_guard<std::mutex> g(words_mu_);
        grow_words();
    }
    ~NvlRail() override {
        std::lock_guard<std::mutex> g(mu_);
        for (void *e : free_events_) gpu::event_destroy(e);
        const int prev = gpu::current_device();
        gpu::set_device(dev_);
        for (auto &sl : word_slabs_) {
            gpu::device_free(sl.first);
            gpu::host_free(sl.second);
        }
        if (prev >= 0) gpu::set_device(prev);
    }

    // Status words (device) and completion words (host-mapped) of this
    // rail's QPs, 64 bytes each, carved from slabs allocated when the rail
    // opens. A QP is created on the accept thread while the process's own
    // device work may be queued behind a collective that waits for this very
    // handshake; taking a slot makes no allocation call there that could
    // wait on the device (cudaMalloc/cudaFree can).
    bool take_words(uint32_t **status, uint64_t **done) {
        std::lock_guard<std::mutex> g(words_mu_);
        if (free_words_.empty() && !grow_words()) return false;
        *status = free_words_.back().first;
        *done = free_words_.back().second;
        free_words_.pop_back();
        return true;
    }
    void give_words(uint32_t *status, uint64_t *done) {
        std::lock_guard<std::mutex> g(words_mu_);
        free_words_.emplace_back(status, done);
    }
    const std::string &name() const override { return name_; }
    std::string gid() const override { return gid_; }
    int numa_node() const override { return numa_; }
    std::string pci_path() const override { return pci_path_; }
    int gpu_ordinal() const override { return dev_; }

    int register_memory(void *addr, size_t len, MemKey *out) override {
        uint32_t key = 0;
        int e = Registry::get().add(addr, len, &key);
        if (e) return e;
        out->lkey = out->rkey = key;
        return 0;
    }
    int deregister_memory(void *, const MemKey &key) override { return Registry::get().remove(key.lkey); }

    std::unique_ptr<QueuePair> create_qp() override {
        std::lock_guard<std::mutex> g(mu_);
        auto qp = std::make_unique<NvlQp>(this, next_qpn_++);
        qps_.push_back(qp.get());
        return qp;
    }
    void forget(NvlQp *qp) {
        std::lock_guard<std::mutex> g(mu_);
        qps_.erase(std::remove(qps_.begin(), qps_.end(), qp), qps_.end());
    }

    int poll(WorkCompletion *out, int max) override {
        std::lock_guard<std::mutex> g(mu_);
        if (cq_.size() < static_cast<size_t>(max))
            for (NvlQp *qp : qps_) qp->reap(&cq_);
        int n = 0;
        while (n < max && !cq_.empty()) {
            out[n++] = cq_.front();
            cq_.pop_front();
        }
        return n;
    }

    size_t preferred_chunk(const Config &cfg) const override {
        return cfg.max_rdma_transfer_size_set ? cfg.max_rdma_transfer_size : cfg.nvl_chunk_size;
    }
    size_t preferred_outstanding(const Config &cfg) const override {
        return cfg.max_outstanding_set ? cfg.max_outstanding_per_qp : cfg.nvl_outstanding_per_qp;
    }
    size_t max_fanout() const override { return kern::kMaxFanoutDsts; }
    bool supports_paged() const override { return true; }
    size_t fanout_alignment() const override { return 16; }
    int set_multicast(const MemKey &key, uintptr_t uc, size_t len, uintptr_t mc, uint64_t token,
                      int members) override {
        return Registry::get().set_multicast(key.lkey, uc, len, mc, token, members);
    }
    int set_stream(void *stream) override {
        // A stream belongs to one device: only that device's rail adopts it.
        if (stream && gpu::stream_device(stream) != dev_) return 0;
        std::lock_guard<std::mutex> g(mu_);
        override_stream_ = stream;
        return 0;
    }
    void set_qos_gate(const uint32_t *gate, uint64_t budget_ns) override {
        std::lock_guard<std::mutex> g(mu_);
        qos_gate_ = gate;
        qos_budget_ns_ = gate ? budget_ns : 0;
    }

    // Launch geometry: a copy touching host memory is PCIe-bound: 2 CTAs
    // per QP already saturate a Gen5 x16 link (measured: 4 x 1 GiB PUT/GET
    // at 51.6-51.9 GB/s for 2..32 CTAs), so it gets 4 — fewer SMs held and
    // fewer loads queued ahead of a concurrent H2D gather. Device-to-device
    // copies share the GPU among the QPs (or take all of it on one caller
    // stream).
    int ctas_for(bool host) const {
        if (cfg_.nvl_ctas_per_qp > 0) return cfg_.nvl_ctas_per_qp;
        if (host) return sms_ < 4 ? sms_ : 4;
        if (override_stream_) return sms_;
        int q = static_cast<int>(cfg_.qps_per_connection);
        int c = q > 0 ? sms_ / q : sms_;
        return c < 1 ? 1 : c;
    }
    void *take_event() {
        if (!free_events_.empty()) {
            void *e = free_events_.back();
            free_events_.pop_back();
            return e;
        }
        return gpu::event_create(dev_);
    }
    void give_event(void *e) { free_events_.push_back(e); }

    std::mutex mu_;
    int dev_;
    void *override_stream_ = nullptr;
    const uint32_t *qos_gate_ = nullptr;  // device QoS gate for H2D copies
    uint64_t qos_budget_ns_ = 0;
    std::deque<WorkCompletion> cq_;

 private:
    const Config &cfg_;
    std::string name_, gid_, pci_path_;
    int numa_ = 0;
    int sms_ = 0;
    uint32_t next_qpn_ = 1;
    std::vector<NvlQp *> qps_;
    std::vector<void *> free_events_;

    static constexpr size_t kWordSlots = 256;  // QPs per slab
    bool grow_words() {  // caller holds words_mu_
        const int prev = gpu::current_device();
        gpu::set_device(dev_);
        auto *d = static_cast<char *>(gpu::device_alloc(kWordSlots * 64));
        auto *h = static_cast<char *>(gpu::host_alloc_mapped(kWordSlots * 64));
        bool ok = d && h && gpu::memset_device(d, 0, kWordSlots * 64) == 0;
        if (prev >= 0) gpu::set_device(prev);
        if (!ok) {
            gpu::device_free(d);
            gpu::host_free(h);
            return false;
        }
        std::memset(h, 0, kWordSlots * 64);
        word_slabs_.emplace_back(d, h);
        for (size_t i = kWordSlots; i-- > 0;)
            free_words_.emplace_back(reinterpret_cast<uint32_t *>(d + i * 64), reinterpret_cast<uint64_t *>(h + i * 64));
        return true;
    }
    std::mutex words_mu_;
    std::vector<std::pair<char *, char *>> word_slabs_;
    std::vector<std::pair<uint32_t *, uint64_t *>> free_words_;
};

NvlQp::NvlQp(NvlRail *rail, uint32_t qpn) : rail_(rail), qpn_(qpn) {
    stream_ = gpu::stream_create(rail_->dev_);
    if (!rail_->take_words(&status_, &done_word_)) {
        status_ = nullptr;
        done_word_ = nullptr;
        return;
    }
    // A recycled slot starts from zero: the status word and last-CTA
    // counter on the device (zeroed on this QP's own non-blocking stream,
    // which then drains, so launches on any stream see it), the completion
    // word on the host.
    int prev = gpu::current_device();
    gpu::set_device(rail_->dev_);
    if (stream_ && gpu::memset_device_async(status_, 0, 64, stream_) == 0) gpu::stream_sync(stream_);
    if (prev >= 0) gpu::set_device(prev);
    __atomic_store_n(done_word_, 0ull, __ATOMIC_RELEASE);
}

NvlQp::~NvlQp() {
    if (stream_) gpu::stream_sync(stream_);
    {
        // Launches may sit on a caller stream: wait for each (they are
        // bounded) before the words they write are freed.
        std::lock_guard<std::mutex> g(rail_->mu_);
        for (auto &f : inflight_) {
            gpu::event_sync(f.event);
            rail_->give_event(f.event);
        }
        inflight_.clear();
    }
    rail_->forget(this);
    gpu::stream_destroy(stream_);
    if (status_) rail_->give_words(status_, done_word_);
}

int NvlQp::to_rtr(const EndpointInfo &remote) {
    std::string boot;
    long pid = -1;
    int dev = -1;
    if (!parse_gid(remote.gid, &boot, &pid, &dev) || boot != boot_tag()) {
        MPCOMM_LOG_WARN("MPComm[nvl]: peer %s is not an nvl rail on this host\n", remote.gid.c_str());
        return MPCOMM_ERR_CONNECTION;
    }
    if (pid == getpid() && dev != rail_->dev_) {
        int e = gpu::enable_peer_access(rail_->dev_, dev);
        if (e != 0) {
            MPCOMM_LOG_WARN("MPComm[nvl]: no peer access %d->%d\n", rail_->dev_, dev);
            return MPCOMM_ERR_CONNECTION;
        }
    }
    remote_ = remote;
    remote_pid_ = pid;
    remote_dev_ = dev;
    state_ = QpState::kRtr;
    return 0;
}

int NvlQp::to_err() {
    state_ = QpState::kErr;
    std::lock_guard<std::mutex> g(rail_->mu_);
    for (size_t i = 0; i < pending_ids_.size(); ++i)
        rail_->cq_.push_back(WorkCompletion{pending_ids_[i], kWcFlushErr, 0});
    pending_.clear();
    pending_ids_.clear();
    pending_lens_.clear();
    for (auto &pf : pending_fanout_) rail_->cq_.push_back(WorkCompletion{pf.wr_id, kWcFlushErr, 0});
    pending_fanout_.clear();
    for (auto &pp : pending_paged_) rail_->cq_.push_back(WorkCompletion{pp.w.wr_id, kWcFlushErr, 0});
    pending_paged_.clear();
    for (auto &f : inflight_) f.failed = true;
    return 0;
}

int NvlQp::post(const WorkRequest *wrs, size_t n) {
    QpState s = state_.load();
    if (s != QpState::kRts && s != QpState::kErr) return MPCOMM_ERR_CONNECTION;
    std::lock_guard<std::mutex> g(rail_->mu_);
    // Peer liveness, checked on the host before anything is launched at the
    // peer's memory: once its process is gone, WRs complete with
    // retry-exceeded and the QP enters the error state (RC semantics).
    if (s == QpState::kRts && remote_pid_ > 0 && remote_pid_ != getpid() &&
        kill(static_cast<pid_t>(remote_pid_), 0) != 0 && errno == ESRCH) {
        MPCOMM_LOG_WARN("MPComm[nvl]: peer process %ld is gone; QP %u on %s -> error\n", remote_pid_, qpn_,
                        rail_->name().c_str());
        for (size_t i = 0; i < n; ++i) rail_->cq_.push_back(WorkCompletion{wrs[i].wr_id, kWcRetryExcErr, 0});
        state_ = QpState::kErr;
        return 0;
    }
    for (size_t i = 0; i < n; ++i) {
        const WorkRequest &wr = wrs[i];
        if (s == QpState::kErr) {
            rail_->cq_.push_back(WorkCompletion{wr.wr_id, kWcFlushErr, 0});
            continue;
        }
        Region lr;
        if (!Registry::get().lookup(wr.lkey, &lr) || wr.local_addr < lr.addr ||
            wr.local_addr + wr.length > lr.addr + lr.len) {
            rail_->cq_.push_back(WorkCompletion{wr.wr_id, kWcLocProtErr, 0});
            continue;
        }
        uintptr_t rptr = 0;
        bool remote_host = false;
        const int st = resolve_remote(wr.rkey, wr.remote_addr, wr.length, &rptr, &remote_host, nullptr);
        if (st != kWcSuccess) {
            rail_->cq_.push_back(WorkCompletion{wr.wr_id, st, 0});
            continue;
        }
        if (lr.device && lr.dev != rail_->dev_) gpu::enable_peer_access(rail_->dev_, lr.dev);
        kern::CopyDesc d;
        if (wr.op == Opcode::kWrite) {
            d.src = reinterpret_cast<const void *>(wr.local_addr);
            d.dst = reinterpret_cast<void *>(rptr);
        } else {
            d.src = reinterpret_cast<const void *>(rptr);
            d.dst = reinterpret_cast<void *>(wr.local_addr);
        }
        d.bytes = wr.length;
        pending_.push_back(d);
        pending_ids_.push_back(wr.wr_id);
        pending_lens_.push_back(wr.length);
        pending_host_ |= remote_host || !lr.device;
        pending_h2d_ |= wr.op == Opcode::kRead && remote_host && lr.device;
    }
    return 0;
}

int NvlQp::resolve_remote(uint32_t rkey, uintptr_t raddr, size_t len, uintptr_t *out, bool *host, McInfo *mc) {
    *host = false;
    if (remote_pid_ == getpid()) {
        Region rr;
        if (!Registry::get().lookup(rkey, &rr) || raddr < rr.addr || raddr + len > rr.addr + rr.len)
            return kWcRemAccessErr;
        if (rr.device && rr.dev != rail_->dev_) gpu::enable_peer_access(rail_->dev_, rr.dev);
        *out = raddr;
        *host = !rr.device;
        if (mc) {
            mc->token = rr.mc_token;
            mc->members = rr.mc_members;
            mc->base = rr.addr;
        }
        return kWcSuccess;
    }
    return RemoteMaps::get().resolve(remote_pid_, rkey, raddr, len, rail_->dev_, out, host, mc);
}

int NvlQp::describe_remote(uint32_t rkey, uintptr_t raddr, size_t len, McInfo *mc) {
    if (remote_pid_ == getpid()) {
        Region rr;
        if (!Registry::get().lookup(rkey, &rr) || raddr < rr.addr || raddr + len > rr.addr + rr.len)
            return kWcRemAccessErr;
        mc->token = rr.mc_token;
        mc->members = rr.mc_members;
        mc->base = rr.addr;
        return kWcSuccess;
    }
    return RemoteMaps::get().describe(remote_pid_, rkey, raddr, len, mc);
}

// One-to-many WRITE. Every target QP is a QP of this rail (one per
// destination connection); each resolves its own peer's range. The bytes go
// out in one gather_bcast launch that reads each source tile once: as
// multicast stores when the destinations are exactly the other members of
// one NVLS group at a common offset (and this process holds the group's
// multicast mapping), else as bulk stores to each destination (<= 8).
int NvlQp::post_fanout(const WorkRequest &wr, const FanoutTarget *targets, size_t n, void *h2d_window) {
    if (n == 0 || n > static_cast<size_t>(kern::kMaxFanoutDsts) || wr.op != Opcode::kWrite ||
        (wr.local_addr | wr.length) & 15u)
        return MPCOMM_ERR_INVALID_ARG;
    for (size_t i = 0; i < n; ++i) {
        auto *q = dynamic_cast<NvlQp *>(targets[i].qp);
        if (!q || q->rail_ != rail_ || (targets[i].remote_addr & 15u)) return MPCOMM_ERR_INVALID_ARG;
    }
    std::lock_guard<std::mutex> g(rail_->mu_);
    auto fail = [&](int st) {
        rail_->cq_.push_back(WorkCompletion{wr.wr_id, st, 0});
        if (h2d_window) __atomic_store_n(&static_cast<kern::H2DWindow *>(h2d_window)->armed, 0u, __ATOMIC_RELEASE);
        return 0;
    };
    for (size_t i = 0; i < n; ++i) {
        auto *q = static_cast<NvlQp *>(targets[i].qp);
        const QpState qs = q->state_.load();
        if (qs == QpState::kErr) return fail(kWcFlushErr);
        if (qs != QpState::kRts) return MPCOMM_ERR_CONNECTION;
        if (q->remote_pid_ > 0 && q->remote_pid_ != getpid() &&
            kill(static_cast<pid_t>(q->remote_pid_), 0) != 0 && errno == ESRCH) {
            MPCOMM_LOG_WARN("MPComm[nvl]: peer process %ld is gone; QP %u on %s -> error\n", q->remote_pid_,
                            q->qpn_, rail_->name().c_str());
            q->state_ = QpState::kErr;
            return fail(kWcRetryExcErr);
        }
    }
    Region lr;
    if (!Registry::get().lookup(wr.lkey, &lr) || wr.local_addr < lr.addr ||
        wr.local_addr + wr.length > lr.addr + lr.len)
        return fail(kWcLocProtErr);
    if (lr.device && lr.dev != rail_->dev_) gpu::enable_peer_access(rail_->dev_, lr.dev);
    PendingFanout f;
    f.src = reinterpret_cast<const void *>(wr.local_addr);
    f.mc = nullptr;
    f.bytes = wr.length;
    f.wr_id = wr.wr_id;
    f.win = static_cast<kern::H2DWindow *>(h2d_window);
    // Pass 1: multicast identity of every target (nothing mapped yet; a
    // group copy may be a VMM allocation that CUDA IPC cannot open).
    uint64_t token = 0;
    int members = 0;
    uintptr_t offset = 0;
    bool same_group = true;
    std::set<std::pair<long, uintptr_t>> owners;  // distinct group copies among the targets
    for (size_t i = 0; i < n; ++i) {
        auto *q = static_cast<NvlQp *>(targets[i].qp);
        McInfo mc;
        const int st = q->describe_remote(targets[i].rkey, targets[i].remote_addr, wr.length, &mc);
        if (st != kWcSuccess) return fail(st);
        const uintptr_t off = targets[i].remote_addr - mc.base;
        if (i == 0) {
            token = mc.token;
            members = mc.members;
            offset = off;
        }
        same_group &= mc.token != 0 && mc.token == token && mc.members == members && off == offset;
        owners.emplace(q->remote_pid_, mc.base);
    }
    same_group &= owners.size() == n;
    // Multicast reaches every member, the sending GPU's own copy included:
    // used only when the targets are exactly the members other than this
    // process's copy, and the source does not overlap that copy's target
    // range except by being it (its multicast store would overwrite bytes
    // still to be read).
    Region mine;
    if (same_group && static_cast<int>(n) + 1 == members && Registry::get().find_multicast(token, &mine) &&
        mine.dev == rail_->dev_ && offset + wr.length <= mine.len) {
        const uintptr_t own = mine.addr + offset;
        const bool overlap = wr.local_addr < own + wr.length && own < wr.local_addr + wr.length;
        if (!overlap || wr.local_addr == own) f.mc = reinterpret_cast<void *>(mine.mc_addr + offset);
    }
    // Pass 2 (P2P sink): each destination mapped on this rail's GPU.
    if (!f.mc) {
        for (size_t i = 0; i < n; ++i) {
            auto *q = static_cast<NvlQp *>(targets[i].qp);
            uintptr_t ptr = 0;
            bool host = false;
            const int st = q->resolve_remote(targets[i].rkey, targets[i].remote_addr, wr.length, &ptr, &host, nullptr);
            if (st != kWcSuccess) return fail(st);
            f.dsts.push_back(reinterpret_cast<void *>(ptr));
        }
    }
    pending_fanout_.push_back(std::move(f));
    return 0;
}

// Paged WRITE: the pages are read by this rail's GPU (from mapped host DRAM
// or device memory) into shared memory and stored straight into the peer's
// range by one launch (the fused PXN gather + forward).
int NvlQp::post_paged(const PagedWrite &w) {
    if (!w.pool || !w.indices || w.count == 0 || w.page_bytes == 0) return MPCOMM_ERR_INVALID_ARG;
    QpState s = state_.load();
    if (s != QpState::kRts && s != QpState::kErr) return MPCOMM_ERR_CONNECTION;
    std::lock_guard<std::mutex> g(rail_->mu_);
    auto fail = [&](int st) {
        rail_->cq_.push_back(WorkCompletion{w.wr_id, st, 0});
        if (w.h2d_window) __atomic_store_n(&static_cast<kern::H2DWindow *>(w.h2d_window)->armed, 0u, __ATOMIC_RELEASE);
        return 0;
    };
    if (s == QpState::kErr) return fail(kWcFlushErr);
    if (remote_pid_ > 0 && remote_pid_ != getpid() && kill(static_cast<pid_t>(remote_pid_), 0) != 0 &&
        errno == ESRCH) {
        state_ = QpState::kErr;
        return fail(kWcRetryExcErr);
    }
    uintptr_t dst = 0;
    bool host = false;
    const size_t bytes = static_cast<size_t>(w.count) * w.page_bytes;
    const int st = resolve_remote(w.rkey, w.remote_addr, bytes, &dst, &host, nullptr);
    if (st != kWcSuccess) return fail(st);
    pending_paged_.push_back(PendingPaged{w, reinterpret_cast<void *>(dst)});
    return 0;
}

void NvlQp::flush() {
    std::lock_guard<std::mutex> g(rail_->mu_);
    if (pending_.empty() && pending_fanout_.empty() && pending_paged_.empty()) return;
    nvtx::Range range("mpcomm::nvl_doorbell");
    gpu::set_device(rail_->dev_);
    void *stream = rail_->override_stream_ ? rail_->override_stream_ : stream_;
    const int ctas = rail_->ctas_for(pending_host_);
    size_t i = 0;
    while (i < pending_.size()) {
        size_t n = pending_.size() - i;
        if (n > static_cast<size_t>(kern::kMaxCopyDescs)) n = kern::kMaxCopyDescs;
        Inflight f;
        f.event = nullptr;
        f.failed = false;
        f.seq = ++seq_;
        f.wr_ids.assign(pending_ids_.begin() + i, pending_ids_.begin() + i + n);
        f.lens.assign(pending_lens_.begin() + i, pending_lens_.begin() + i + n);
        const bool gated = pending_h2d_ && rail_->qos_gate_;
        int e = done_word_ ? 0 : -1;
        if (e == 0)
            e = kern::copy_batch(pending_.data() + i, static_cast<int>(n), ctas, stream, status_, nullptr,
                                 kern::kModeAuto, gated ? rail_->qos_gate_ : nullptr,
                                 gated ? rail_->qos_budget_ns_ : 0, done_word_, f.seq, status_ + 4);
        if (e == 0) {
            f.event = rail_->take_event();
            if (!f.event || gpu::event_record(f.event, stream) != 0) e = -1;
        }
        if (e != 0) {
            MPCOMM_LOG_ERROR("MPComm[nvl]: copy launch failed on %s: %s\n", rail_->name().c_str(),
                             e > 0 ? gpu::error_string(e) : "event");
            for (size_t k = 0; k < n; ++k)
                rail_->cq_.push_back(WorkCompletion{f.wr_ids[k], kWcGeneralErr, 0});
            if (f.event) rail_->give_event(f.event);
        } else {
            f.launched = std::chrono::steady_clock::now();
            inflight_.push_back(std::move(f));
        }
        i += n;
    }
    pending_.clear();
    pending_ids_.clear();
    pending_lens_.clear();
    pending_host_ = false;
    pending_h2d_ = false;
    for (auto &pf : pending_fanout_) {
        Inflight f;
        f.event = nullptr;
        f.failed = false;
        f.seq = ++seq_;
        f.wr_ids.assign(1, pf.wr_id);
        f.lens.assign(1, pf.bytes);
        uint64_t *flag = done_word_;
        int e = done_word_ ? 0 : -1;
        if (e == 0)
            e = kern::gather_bcast(pf.src, 0, nullptr, 1, pf.bytes, pf.mc, pf.dsts.data(),
                                   static_cast<int>(pf.dsts.size()), nullptr, &flag, 1, f.seq, status_ + 4, 0, stream,
                                   status_, nullptr, pf.win);
        if (e == 0) {
            f.event = rail_->take_event();
            if (!f.event || gpu::event_record(f.event, stream) != 0) e = -1;
        }
        if (e != 0) {
            MPCOMM_LOG_ERROR("MPComm[nvl]: fan-out launch failed on %s: %s\n", rail_->name().c_str(),
                             e > 0 ? gpu::error_string(e) : "event");
            rail_->cq_.push_back(WorkCompletion{pf.wr_id, kWcGeneralErr, 0});
            if (f.event) rail_->give_event(f.event);
            if (pf.win) __atomic_store_n(&pf.win->armed, 0u, __ATOMIC_RELEASE);
        } else {
            f.launched = std::chrono::steady_clock::now();
            inflight_.push_back(std::move(f));
        }
    }
    pending_fanout_.clear();
    for (auto &pp : pending_paged_) {
        Inflight f;
        f.event = nullptr;
        f.failed = false;
        f.seq = ++seq_;
        f.wr_ids.assign(1, pp.w.wr_id);
        f.lens.assign(1, pp.w.count * pp.w.page_bytes);
        auto *win = static_cast<kern::H2DWindow *>(pp.w.h2d_window);
        int e = done_word_ ? 0 : -1;
        if (e == 0)
            e = kern::pxn_gather_forward(reinterpret_cast<const void *>(pp.w.pool),
                                         static_cast<int64_t>(pp.w.pool_pages), pp.w.indices, pp.dst, pp.w.count,
                                         pp.w.page_bytes, 0, stream, status_, done_word_, f.seq, status_ + 4, nullptr,
                                         win);
        if (e == 0) {
            f.event = rail_->take_event();
            if (!f.event || gpu::event_record(f.event, stream) != 0) e = -1;
        }
        if (e != 0) {
            MPCOMM_LOG_ERROR("MPComm[nvl]: paged launch failed on %s: %s\n", rail_->name().c_str(),
                             e > 0 ? gpu::error_string(e) : "event");
            rail_->cq_.push_back(WorkCompletion{pp.w.wr_id, kWcGeneralErr, 0});
            if (f.event) rail_->give_event(f.event);
            if (win) __atomic_store_n(&win->armed, 0u, __ATOMIC_RELEASE);
        } else {
            f.launched = std::chrono::steady_clock::now();
            inflight_.push_back(std::move(f));
        }
    }
    pending_paged_.clear();
}

void NvlQp::reap(std::deque<WorkCompletion> *cq) {
    if (inflight_.empty()) return;
    uint64_t done = __atomic_load_n(done_word_, __ATOMIC_ACQUIRE);
    while (!inflight_.empty()) {
        Inflight &f = inflight_.front();
        int q = 1;
        if (f.seq > done && !f.failed) {
            // Not signalled yet: consult the event only now and then.
            const auto now = std::chrono::steady_clock::now();
            if (now - f.launched < kEventCheckAfter || now < next_check_) return;
            next_check_ = now + kEventCheckAfter;
            gpu::set_device(rail_->dev_);  // the event belongs to this rail's device
            q = gpu::event_query(f.event);
            if (q < 0)
                MPCOMM_LOG_WARN("MPComm[nvl]: launch %lu on %s failed: %s\n", static_cast<unsigned long>(f.seq),
                                rail_->name().c_str(), gpu::error_string(-q));
            if (q == 0) return;
            // The event completed, so the kernel's last store (the done
            // word) has been issued: allow it a moment to land, then treat
            // a missing word as a failed launch.
            for (int spin = 0; q > 0 && spin < 1000; ++spin) {
                done = __atomic_load_n(done_word_, __ATOMIC_ACQUIRE);
                if (f.seq <= done) break;
                cpu_relax();
            }
            if (q > 0 && f.seq > done) {
                MPCOMM_LOG_WARN("MPComm[nvl]: launch %lu on %s completed without its done word\n",
                                static_cast<unsigned long>(f.seq), rail_->name().c_str());
                q = -1;
            }
        }
        bool bad = f.failed || q < 0;
        if (!bad) {
            // A kernel can only have timed out if it ran at least the wait
            // budget; only then is the device status word read back.
            double ran = std::chrono::duration<double>(std::chrono::steady_clock::now() - f.launched).count();
            if (ran * 1e9 >= 0.9 * static_cast<double>(kern::wait_budget_ns())) {
                uint32_t st = 0;
                gpu::set_device(rail_->dev_);
                gpu::copy_d2h_sync(&st, status_, sizeof(st));
                if (st) {
                    bad = true;
                    gpu::memset_device(status_, 0, sizeof(uint32_t));
                }
            }
        }
        for (size_t k = 0; k < f.wr_ids.size(); ++k)
            cq->push_back(WorkCompletion{f.wr_ids[k], bad ? kWcGeneralErr : kWcSuccess,
                                         bad ? 0u : f.lens[k]});
        rail_->give_event(f.event);
        inflight_.pop_front();
    }
}

class NvlBackend final : public Backend {
 public:
    const char *name() const override { return "nvl"; }
    int open(const Config &cfg, const std::vector<std::string> &filter,
             std::vector<std::unique_ptr<Rail>> *rails) override {
        int n = gpu::device_count();
        for (int d = 0; d < n; ++d) {
            std::string nm = "nvl_" + std::to_string(d);
            if (!filter.empty()) {
                bool ok = false;
                for (auto &f : filter) ok |= (f == nm);
                if (!ok) continue;
            }
            rails->push_back(std::make_unique<NvlRail>(d, cfg));
        }
        return rails->empty() ? MPCOMM_ERR_DEVICE : MPCOMM_SUCCESS;
    }
};

}  // namespace

std::unique_ptr<Backend> make_nvl_backend() { return std::make_unique<NvlBackend>(); }
int nvl_device_count() { return gpu::device_count(); }

}  // namespace fabric
}  // namespace mpcomm
