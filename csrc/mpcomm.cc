// Public facade: MPComm forwards to MPComm::Impl (pimpl keeps the ABI of
// the class stable; reference src/mpcomm.cpp:7516-7965).
#include "mpcomm.h"

#include "engine/impl.h"
#include "kernels/launch.h"
#include "parallel/mcgroup.h"

namespace mpcomm {

MPComm::MPComm() : impl_(new Impl()) {}
MPComm::~MPComm() = default;
MPComm::MPComm(MPComm &&) noexcept = default;
MPComm &MPComm::operator=(MPComm &&) noexcept = default;

int MPComm::init(const std::string &id, const std::string &devs, int port) { return impl_->init(id, devs, port); }
void MPComm::shutdown() { impl_->shutdown(); }
int MPComm::registerMemory(void *a, size_t l) { return impl_->registerMemory(a, l); }
int MPComm::unregisterMemory(void *a) { return impl_->unregisterMemory(a); }
int MPComm::connect(const std::string &id, const std::string &addr, int port) {
    return impl_->connect(id, addr, port);
}
int MPComm::startAcceptThread() { return impl_->startAcceptThread(); }
void MPComm::stopAcceptThread() { impl_->stopAcceptThread(); }
int MPComm::updateRemoteMemoryInfo(const std::string &id, const std::vector<uint32_t> &rkeys) {
    return impl_->updateRemoteMemoryInfo(id, rkeys);
}
int MPComm::publishBuffer(void *a, size_t l, int numa) { return impl_->publishBuffer(a, l, numa); }
int MPComm::unpublishBuffer(void *a) { return impl_->unpublishBuffer(a); }
void MPComm::unpublishAllBuffers() { impl_->unpublishAllBuffers(); }
int MPComm::queryRemoteBuffer(const std::string &id, const std::string &addr, int port,
                              RemoteBufferInfo &out) {
    return impl_->queryRemoteBuffer(id, addr, port, out);
}
int MPComm::queryRemoteBufferByNuma(const std::string &id, const std::string &addr, int port, int numa,
                                    RemoteBufferEntry &out) {
    return impl_->queryRemoteBufferByNuma(id, addr, port, numa, out);
}
const PublishedBufferInfo *MPComm::getPublishedBufferInfo() const { return impl_->getPublishedBufferInfo(); }
size_t MPComm::getPublishedBufferCount() const { return impl_->getPublishedBufferCount(); }
uint32_t MPComm::getRkey(size_t nic, void *addr) const { return impl_->getRkey(nic, addr); }

TransferHandle MPComm::scatterAsync(uintptr_t local, const std::vector<std::string> &hosts,
                                    const std::vector<uintptr_t> &raddrs, const std::vector<size_t> &lens) {
    return impl_->submit(local, hosts, raddrs, lens, Direction::kScatter);
}
TransferHandle MPComm::gatherAsync(uintptr_t local, const std::vector<std::string> &hosts,
                                   const std::vector<uintptr_t> &raddrs, const std::vector<size_t> &lens) {
    return impl_->submit(local, hosts, raddrs, lens, Direction::kGather);
}
TransferHandle MPComm::broadcastAsync(uintptr_t local, size_t len, const std::vector<std::string> &hosts,
                                      const std::vector<uintptr_t> &raddrs) {
    if (hosts.empty() || raddrs.size() != hosts.size() || len == 0) return INVALID_TRANSFER_HANDLE;
    return impl_->submit(local, hosts, raddrs, std::vector<size_t>(hosts.size(), len), Direction::kBroadcast);
}
TransferHandle MPComm::putPagesAsync(uintptr_t dram_dev_ptr, const int64_t *indices, int num_blocks, int block_size,
                                     const std::string &host, uintptr_t raddr) {
    return impl_->submitPaged(dram_dev_ptr, indices, num_blocks, block_size, host, raddr);
}
TransferHandle MPComm::putAsync(uintptr_t local, const std::string &host, uintptr_t raddr, size_t len) {
    if (len == 0) return INVALID_TRANSFER_HANDLE;
    return impl_->submit(local, {host}, {raddr}, {len}, Direction::kScatter);
}
TransferHandle MPComm::getAsync(uintptr_t local, const std::string &host, uintptr_t raddr, size_t len) {
    if (len == 0) return INVALID_TRANSFER_HANDLE;
    return impl_->submit(local, {host}, {raddr}, {len}, Direction::kGather);
}
bool MPComm::isTransferComplete(TransferHandle h) { return impl_->isTransferComplete(h); }
int MPComm::waitTransfer(TransferHandle h, int timeout_ms) { return impl_->waitTransfer(h, timeout_ms); }
TransferResult MPComm::getTransferResult(TransferHandle h) { return impl_->getTransferResult(h); }
void MPComm::releaseTransfer(TransferHandle h) { impl_->releaseTransfer(h); }

size_t MPComm::getNumNics() const { return impl_->numNics(); }
const std::string &MPComm::getLocalHostId() const { return impl_->hostId(); }
int MPComm::getTcpPort() const { return impl_->tcpPort(); }
std::string MPComm::getGid(size_t i) const { return impl_->gid(i); }
std::string MPComm::getDeviceName(size_t i) const { return impl_->deviceName(i); }
std::vector<std::string> MPComm::getActiveDevices() const { return impl_->activeDevices(); }
const char *MPComm::getNicFilterEnvVarName() { return "MPCOMM_NIC_FILTER"; }
size_t MPComm::getMaxRdmaTransferSize() const { return impl_->maxRdmaTransferSize(); }

void MPComm::setNicThrottle(size_t o, size_t c) { impl_->setNicThrottle(o, c); }
void MPComm::clearNicThrottle() { impl_->clearNicThrottle(); }
void MPComm::enableH2DQoS(uint64_t r, uint64_t b) { impl_->enableH2DQoS(r, b); }
void MPComm::setH2DQoSPolicy(uint64_t r, uint64_t b) { impl_->setH2DQoSPolicy(r, b); }
bool MPComm::isH2DQoSEnabled() const { return impl_->isH2DQoSEnabled(); }
bool MPComm::getLastH2DWindow(int gpu, uint64_t *b, uint64_t *e) const { return impl_->lastH2DWindow(gpu, b, e); }
int MPComm::openQosChannel(const std::string &h) { return impl_->openQosChannel(h); }
int MPComm::closeQosChannel(const std::string &h) { return impl_->closeQosChannel(h); }
int MPComm::sendQosPolicy(const std::string &h, int gpu, uint64_t rate, uint64_t burst) {
    return impl_->sendQosPolicy(h, gpu, rate, burst, false);
}
int MPComm::clearQosPolicy(const std::string &h, int gpu) { return impl_->sendQosPolicy(h, gpu, 0, 0, true); }
std::vector<MPComm::RemoteQosPolicy> MPComm::getRemoteQosPolicies() const {
    std::vector<RemoteQosPolicy> out;
    for (auto &v : impl_->remoteQosPolicies()) out.push_back(RemoteQosPolicy{v.peer, v.gpu, v.rate, v.burst, v.generation});
    return out;
}
uint64_t MPComm::getRemoteQosDeferCount() const { return impl_->remoteQosDefers(); }
void MPComm::disableH2DQoS() { impl_->disableH2DQoS(); }
uint64_t MPComm::getNicCompletedBytes() const { return impl_->getNicCompletedBytes(); }
std::vector<uint64_t> MPComm::getRailCompletedBytes() const { return impl_->railCompletedBytes(); }
std::vector<MPComm::PcieDomainStats> MPComm::getPcieDomainStats() const { return impl_->getPcieDomainStats(); }
void MPComm::resetPcieDomainStats() { impl_->resetPcieDomainStats(); }
bool MPComm::isPcieDomainStatEnabled() const { return impl_->isPcieDomainStatEnabled(); }
const char *MPComm::getPcieStatEnableEnvVarName() { return "MPCOMM_PCIE_STAT_ENABLE"; }
bool MPComm::getThrottleLatency(uint64_t *s, uint64_t *w, uint64_t *d, size_t *n) const {
    return impl_->getThrottleLatency(s, w, d, n);
}
size_t MPComm::getQpsPerConnection() const { return impl_->qpsPerConnection(); }
const char *MPComm::getQpsPerConnectionEnvVarName() { return "MPCOMM_QPS_PER_CONNECTION"; }

const std::vector<NumaTopology> &MPComm::getNumaTopology() const { return impl_->numaTopology(); }
const std::vector<NicTopologyInfo> &MPComm::getNicTopology() const { return impl_->nicTopology(); }
int MPComm::getNicNumaNode(const std::string &n) const { return impl_->nicNumaNode(n); }
int MPComm::getNumaNodeForAddr(void *a) const { return impl_->numaNodeForAddr(a); }
std::vector<size_t> MPComm::getLocalNicIndicesForNuma(int n) const { return impl_->localNicsForNuma(n); }
int MPComm::getGpuNumaNode(int g) const { return impl_->gpuNumaNode(g); }

uintptr_t MPComm::mapDRAMtoGPU(void *h, size_t l) { return impl_->mapDRAMtoGPU(h, l); }
int MPComm::unmapDRAMfromGPU(void *h) { return impl_->unmapDRAMfromGPU(h); }
int MPComm::tmaGather(uintptr_t dram, const int64_t *idx, void *dst, int n, int bs, int max_sm, H2DMode mode) {
    return impl_->h2dMove(true, dram, idx, dst, n, bs, max_sm, mode, nullptr);
}
int MPComm::tmaScatter(void *src, const int64_t *idx, uintptr_t dram, int n, int bs, int max_sm, H2DMode mode) {
    return impl_->h2dMove(false, dram, idx, src, n, bs, max_sm, mode, nullptr);
}
int MPComm::tmaGatherOnStream(uintptr_t dram, const int64_t *idx, void *dst, int n, int bs, int max_sm,
                              H2DMode mode, void *stream) {
    return impl_->h2dMove(true, dram, idx, dst, n, bs, max_sm, mode, stream);
}
int MPComm::tmaScatterOnStream(void *src, const int64_t *idx, uintptr_t dram, int n, int bs, int max_sm,
                               H2DMode mode, void *stream) {
    return impl_->h2dMove(false, dram, idx, src, n, bs, max_sm, mode, stream);
}
int MPComm::setFabricStream(void *stream) { return impl_->setFabricStream(stream); }
uint64_t MPComm::getKernelLaunchCount() { return kern::launch_count(); }
std::vector<MPComm::KernelTraceRecord> MPComm::getKernelTrace() {
    std::vector<kern::TraceRecord> raw;
    std::vector<KernelTraceRecord> out;
    if (kern::kernel_trace(&raw) != 0) return out;
    for (const auto &r : raw) out.push_back(KernelTraceRecord{r.seq, r.dev, r.kind ? r.kind : "", r.bytes, r.begin_ns, r.end_ns});
    return out;
}
std::string MPComm::getFabricName() const { return impl_->fabricName(); }
std::vector<MPComm::PcieAffinityCheck> MPComm::getPcieAffinitySelfCheck() const {
    return impl_->pcieAffinitySelfCheck();
}
int MPComm::registerMulticastMemory(void *uc_addr, size_t length, void *mc_addr, uint64_t group_token,
                                    int group_size) {
    return impl_->registerMulticastMemory(uc_addr, length, mc_addr, group_token, group_size);
}
int MPComm::registerMulticastGroup(const MulticastGroup &g) {
    return impl_->registerMulticastMemory(g.uc_addr, g.length, g.mc_addr, g.token, g.members);
}

namespace {
int group_result(int rc, const vmm::McGroup &g, MulticastGroup *out) {
    if (rc != 0) return rc < 0 ? MPCOMM_ERR_CONNECTION : MPCOMM_ERR_DEVICE;
    out->uc_addr = g.uc;
    out->mc_addr = g.mcva;
    out->length = g.size;
    out->token = g.token;
    out->members = g.members;
    out->device = g.dev;
    out->mc_handle = g.mc;
    out->mem_handle = g.mem;
    return MPCOMM_SUCCESS;
}
}  // namespace

int createMulticastGroup(const std::string &name, size_t bytes, int members, MulticastGroup *out, int timeout_ms) {
    if (!out || name.empty() || members < 2 || bytes == 0 || timeout_ms <= 0) return MPCOMM_ERR_INVALID_ARG;
    vmm::McGroup g;
    return group_result(vmm::mc_group_create(name, bytes, members, timeout_ms, &g), g, out);
}
int joinMulticastGroup(const std::string &name, size_t bytes, int members, MulticastGroup *out, int timeout_ms) {
    if (!out || name.empty() || members < 2 || bytes == 0 || timeout_ms <= 0) return MPCOMM_ERR_INVALID_ARG;
    vmm::McGroup g;
    return group_result(vmm::mc_group_join(name, bytes, members, timeout_ms, &g), g, out);
}
int releaseMulticastGroup(MulticastGroup *out) {
    if (!out) return MPCOMM_ERR_INVALID_ARG;
    vmm::McGroup g;
    g.mc = out->mc_handle;
    g.mem = out->mem_handle;
    g.uc = out->uc_addr;
    g.mcva = out->mc_addr;
    g.size = out->length;
    g.dev = out->device;
    const int e = vmm::mc_group_release(&g);
    *out = MulticastGroup{};
    return e ? MPCOMM_ERR_DEVICE : MPCOMM_SUCCESS;
}

}  // namespace mpcomm
