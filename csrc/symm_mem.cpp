// Symmetric-memory bootstrap for one NVSwitch box (N1).
//
// Each rank allocates one physical region with the CUDA virtual-memory API,
// exports it as a POSIX file descriptor, passes the descriptor to every peer over
// an abstract unix socket (SCM_RIGHTS), and maps every peer's region into its own
// address space with read/write access for its GPU.  The NVLS multicast object is
// created by rank 0, shared the same way, joined by every rank's device, bound to a
// second physical allocation per rank and mapped, giving `multimem` addresses.
//
// Replaces the reference's RDMA proxy setup (sparknet/oneshot/_roce_proxy.c:477-729,
// sparknet/oneshot/_proxy.py:71-348): instead of registering pinned host memory
// with an HCA and exchanging rkeys/GIDs, ranks exchange VMM handles and the GPU
// writes peers' memory directly over NVLink.
//
// The driver API is resolved with dlopen at first use, so this module loads on a
// host without a GPU driver (the build host) and fails with a clear message there.
#include "sparknet/symm_mem.h"

#include <cuda.h>
#include <dlfcn.h>
#include <errno.h>
#include <poll.h>
#include <string.h>
#include <sys/socket.h>
#include <sys/un.h>
#include <time.h>
#include <unistd.h>

#include <stdexcept>
#include <string>

namespace sn {

namespace {

struct Driver {
  void* lib = nullptr;
  CUresult (*cuInit)(unsigned);
  CUresult (*cuDeviceGet)(CUdevice*, int);
  CUresult (*cuDeviceGetAttribute)(int*, CUdevice_attribute, CUdevice);
  CUresult (*cuGetErrorString)(CUresult, const char**);
  CUresult (*cuMemGetAllocationGranularity)(size_t*, const CUmemAllocationProp*, CUmemAllocationGranularity_flags);
  CUresult (*cuMemCreate)(CUmemGenericAllocationHandle*, size_t, const CUmemAllocationProp*, unsigned long long);
  CUresult (*cuMemRelease)(CUmemGenericAllocationHandle);
  CUresult (*cuMemExportToShareableHandle)(void*, CUmemGenericAllocationHandle, CUmemAllocationHandleType,
                                           unsigned long long);
  CUresult (*cuMemImportFromShareableHandle)(CUmemGenericAllocationHandle*, void*, CUmemAllocationHandleType);
  CUresult (*cuMemAddressReserve)(CUdeviceptr*, size_t, size_t, CUdeviceptr, unsigned long long);
  CUresult (*cuMemAddressFree)(CUdeviceptr, size_t);
  CUresult (*cuMemMap)(CUdeviceptr, size_t, size_t, CUmemGenericAllocationHandle, unsigned long long);
  CUresult (*cuMemUnmap)(CUdeviceptr, size_t);
  CUresult (*cuMemSetAccess)(CUdeviceptr, size_t, const CUmemAccessDesc*, size_t);
  CUresult (*cuMulticastCreate)(CUmemGenericAllocationHandle*, const CUmulticastObjectProp*);
  CUresult (*cuMulticastAddDevice)(CUmemGenericAllocationHandle, CUdevice);
  CUresult (*cuMulticastBindMem)(CUmemGenericAllocationHandle, size_t, CUmemGenericAllocationHandle, size_t, size_t,
                                 unsigned long long);
  CUresult (*cuMulticastUnbind)(CUmemGenericAllocationHandle, CUdevice, size_t, size_t);
  CUresult (*cuMulticastGetGranularity)(size_t*, const CUmulticastObjectProp*, CUmulticastGranularity_flags);
};

template <typename F>
void bind(Driver& d, F& fn, const char* name) {
  fn = reinterpret_cast<F>(dlsym(d.lib, name));
  if (!fn) throw std::runtime_error(std::string("CUDA driver lacks ") + name);
}

Driver& driver() {
  static Driver d;
  static bool ready = false;
  if (ready) return d;
  d.lib = dlopen("libcuda.so.1", RTLD_NOW | RTLD_GLOBAL);
  if (!d.lib) throw std::runtime_error("libcuda.so.1 not found: symmetric memory needs the NVIDIA driver");
  bind(d, d.cuInit, "cuInit");
  bind(d, d.cuDeviceGet, "cuDeviceGet");
  bind(d, d.cuDeviceGetAttribute, "cuDeviceGetAttribute");
  bind(d, d.cuGetErrorString, "cuGetErrorString");
  bind(d, d.cuMemGetAllocationGranularity, "cuMemGetAllocationGranularity");
  bind(d, d.cuMemCreate, "cuMemCreate");
  bind(d, d.cuMemRelease, "cuMemRelease");
  bind(d, d.cuMemExportToShareableHandle, "cuMemExportToShareableHandle");
  bind(d, d.cuMemImportFromShareableHandle, "cuMemImportFromShareableHandle");
  bind(d, d.cuMemAddressReserve, "cuMemAddressReserve");
  bind(d, d.cuMemAddressFree, "cuMemAddressFree");
  bind(d, d.cuMemMap, "cuMemMap");
  bind(d, d.cuMemUnmap, "cuMemUnmap");
  bind(d, d.cuMemSetAccess, "cuMemSetAccess");
  bind(d, d.cuMulticastCreate, "cuMulticastCreate");
  bind(d, d.cuMulticastAddDevice, "cuMulticastAddDevice");
  bind(d, d.cuMulticastBindMem, "cuMulticastBindMem");
  bind(d, d.cuMulticastUnbind, "cuMulticastUnbind");
  bind(d, d.cuMulticastGetGranularity, "cuMulticastGetGranularity");
  if (d.cuInit(0) != CUDA_SUCCESS) throw std::runtime_error("cuInit failed");
  ready = true;
  return d;
}

void ck(CUresult r, const char* what) {
  if (r == CUDA_SUCCESS) return;
  const char* msg = "unknown";
  driver().cuGetErrorString(r, &msg);
  throw std::runtime_error(std::string(what) + " failed: " + msg + " (" + std::to_string(int(r)) + ")");
}

CUmemAllocationProp device_prop(int device) {
  CUmemAllocationProp p;
  memset(&p, 0, sizeof(p));
  p.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  p.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  p.location.id = device;
  p.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  return p;
}

void map_rw(CUdeviceptr va, size_t bytes, CUmemGenericAllocationHandle h, int device) {
  Driver& d = driver();
  ck(d.cuMemMap(va, bytes, 0, h, 0), "cuMemMap");
  CUmemAccessDesc a;
  memset(&a, 0, sizeof(a));
  a.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  a.location.id = device;
  a.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  const CUresult r = d.cuMemSetAccess(va, bytes, &a, 1);
  if (r != CUDA_SUCCESS) d.cuMemUnmap(va, bytes);  // leave nothing mapped behind the error
  ck(r, "cuMemSetAccess");
}

sockaddr_un abstract_addr(const std::string& name, socklen_t* len) {
  sockaddr_un a;
  memset(&a, 0, sizeof(a));
  a.sun_family = AF_UNIX;
  if (name.size() + 1 > sizeof(a.sun_path)) throw std::invalid_argument("socket name too long");
  a.sun_path[0] = '\0';  // abstract namespace: no file, gone when the process exits
  memcpy(a.sun_path + 1, name.data(), name.size());
  *len = socklen_t(offsetof(sockaddr_un, sun_path) + 1 + name.size());
  return a;
}

double now_s() {
  timespec t;
  clock_gettime(CLOCK_MONOTONIC, &t);
  return t.tv_sec + t.tv_nsec * 1e-9;
}

}  // namespace

// ---------------------------------------------------------------------------
// File-descriptor passing
// ---------------------------------------------------------------------------
int fd_listen(const std::string& name) {
  int s = socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
  if (s < 0) throw std::runtime_error("socket: " + std::string(strerror(errno)));
  socklen_t len;
  sockaddr_un a = abstract_addr(name, &len);
  if (bind(s, reinterpret_cast<sockaddr*>(&a), len) != 0 || listen(s, 64) != 0) {
    int e = errno;
    close(s);
    throw std::runtime_error("bind/listen " + name + ": " + strerror(e));
  }
  return s;
}

void fd_serve(int listener, int fd, int clients, int timeout_ms) {
  double deadline = now_s() + timeout_ms / 1000.0;
  for (int i = 0; i < clients; ++i) {
    pollfd p{listener, POLLIN, 0};
    int left = int((deadline - now_s()) * 1000);
    if (left <= 0 || poll(&p, 1, left) <= 0) throw std::runtime_error("fd_serve: peers did not connect in time");
    int c = accept4(listener, nullptr, nullptr, SOCK_CLOEXEC);
    if (c < 0) throw std::runtime_error("accept: " + std::string(strerror(errno)));
    char byte = 'S';
    iovec iov{&byte, 1};
    char ctl[CMSG_SPACE(sizeof(int))];
    memset(ctl, 0, sizeof(ctl));
    msghdr msg;
    memset(&msg, 0, sizeof(msg));
    msg.msg_iov = &iov;
    msg.msg_iovlen = 1;
    msg.msg_control = ctl;
    msg.msg_controllen = sizeof(ctl);
    cmsghdr* cm = CMSG_FIRSTHDR(&msg);
    cm->cmsg_level = SOL_SOCKET;
    cm->cmsg_type = SCM_RIGHTS;
    cm->cmsg_len = CMSG_LEN(sizeof(int));
    memcpy(CMSG_DATA(cm), &fd, sizeof(int));
    ssize_t n = sendmsg(c, &msg, 0);
    int e = errno;
    close(c);
    if (n != 1) throw std::runtime_error("sendmsg: " + std::string(strerror(e)));
  }
}

int fd_fetch(const std::string& name, int timeout_ms) {
  double deadline = now_s() + timeout_ms / 1000.0;
  for (;;) {
    int s = socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
    if (s < 0) throw std::runtime_error("socket: " + std::string(strerror(errno)));
    socklen_t len;
    sockaddr_un a = abstract_addr(name, &len);
    if (connect(s, reinterpret_cast<sockaddr*>(&a), len) == 0) {
      char byte = 0;
      iovec iov{&byte, 1};
      char ctl[CMSG_SPACE(sizeof(int))];
      msghdr msg;
      memset(&msg, 0, sizeof(msg));
      msg.msg_iov = &iov;
      msg.msg_iovlen = 1;
      msg.msg_control = ctl;
      msg.msg_controllen = sizeof(ctl);
      pollfd p{s, POLLIN, 0};
      int left = int((deadline - now_s()) * 1000);
      if (left <= 0 || poll(&p, 1, left) <= 0) {
        close(s);
        throw std::runtime_error("fd_fetch: no descriptor from " + name);
      }
      ssize_t n = recvmsg(s, &msg, MSG_CMSG_CLOEXEC);
      close(s);
      cmsghdr* cm = CMSG_FIRSTHDR(&msg);
      if (n != 1 || !cm || cm->cmsg_type != SCM_RIGHTS) throw std::runtime_error("fd_fetch: malformed message");
      int fd;
      memcpy(&fd, CMSG_DATA(cm), sizeof(int));
      return fd;
    }
    close(s);
    if (now_s() > deadline) throw std::runtime_error("fd_fetch: cannot connect to " + name);
    usleep(2000);
  }
}

void fd_close(int fd) {
  if (fd >= 0) close(fd);
}

// ---------------------------------------------------------------------------
// Unicast regions
// ---------------------------------------------------------------------------
size_t vmm_granularity(int device) {
  CUmemAllocationProp p = device_prop(device);
  size_t g = 0;
  ck(driver().cuMemGetAllocationGranularity(&g, &p, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED), "granularity");
  return g;
}

int device_attribute(int device, int attr) {
  Driver& d = driver();
  CUdevice dev;
  ck(d.cuDeviceGet(&dev, device), "cuDeviceGet");
  int v = 0;
  ck(d.cuDeviceGetAttribute(&v, CUdevice_attribute(attr), dev), "cuDeviceGetAttribute");
  return v;
}

bool multicast_supported(int device) {
  return device_attribute(device, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED) != 0;
}

LocalRegion::LocalRegion(int device, size_t bytes, size_t align) : device_(device) {
  Driver& d = driver();
  size_t g = vmm_granularity(device);
  if (align > g) g = align;
  bytes_ = (bytes + g - 1) / g * g;
  CUmemAllocationProp p = device_prop(device);
  CUmemGenericAllocationHandle h;
  ck(d.cuMemCreate(&h, bytes_, &p, 0), "cuMemCreate");
  CUdeviceptr va = 0;
  try {  // a constructor that throws runs no destructor: release here what it took
    ck(d.cuMemAddressReserve(&va, bytes_, g, 0, 0), "cuMemAddressReserve");
    map_rw(va, bytes_, h, device);
  } catch (...) {
    if (va) d.cuMemAddressFree(va, bytes_);
    d.cuMemRelease(h);
    throw;
  }
  handle_ = h;
  ptr_ = va;
}

LocalRegion::~LocalRegion() {
  try {
    Driver& d = driver();
    for (auto& m : peers_) {
      d.cuMemUnmap(m.ptr, m.bytes);
      d.cuMemAddressFree(m.ptr, m.bytes);
      d.cuMemRelease(m.handle);
    }
    if (ptr_) {
      d.cuMemUnmap(ptr_, bytes_);
      d.cuMemAddressFree(ptr_, bytes_);
    }
    if (handle_) d.cuMemRelease(handle_);
  } catch (...) {
  }
}

int LocalRegion::export_fd() const {
  int fd = -1;
  ck(driver().cuMemExportToShareableHandle(&fd, handle_, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0),
     "cuMemExportToShareableHandle");
  return fd;
}

uint64_t LocalRegion::map_peer(int fd, size_t bytes) {
  Driver& d = driver();
  CUmemGenericAllocationHandle h;
  ck(d.cuMemImportFromShareableHandle(&h, reinterpret_cast<void*>(static_cast<uintptr_t>(fd)),
                                      CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR),
     "cuMemImportFromShareableHandle");
  CUdeviceptr va = 0;
  try {  // the peer is recorded (and released by the destructor) only once it is mapped
    ck(d.cuMemAddressReserve(&va, bytes, vmm_granularity(device_), 0, 0), "cuMemAddressReserve(peer)");
    map_rw(va, bytes, h, device_);
    peers_.push_back({va, bytes, h});
  } catch (...) {
    if (va) d.cuMemAddressFree(va, bytes);
    d.cuMemRelease(h);
    throw;
  }
  return va;
}

// ---------------------------------------------------------------------------
// Multicast (NVLS)
// ---------------------------------------------------------------------------
Multicast::Multicast(int device, size_t bytes, int ranks) : device_(device), ranks_(ranks) {
  Driver& d = driver();
  CUmulticastObjectProp mp;
  memset(&mp, 0, sizeof(mp));
  mp.numDevices = unsigned(ranks);
  mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  mp.size = bytes;
  size_t g = 0;
  ck(d.cuMulticastGetGranularity(&g, &mp, CU_MULTICAST_GRANULARITY_RECOMMENDED), "cuMulticastGetGranularity");
  size_t ug = vmm_granularity(device);
  if (ug > g) g = ug;
  gran_ = g;
  bytes_ = (bytes + g - 1) / g * g;
  mp.size = bytes_;
  prop_size_ = bytes_;
}

Multicast::~Multicast() {
  try {
    Driver& d = driver();
    CUdevice dev;
    d.cuDeviceGet(&dev, device_);
    if (mc_ptr_) {
      d.cuMemUnmap(mc_ptr_, bytes_);
      d.cuMemAddressFree(mc_ptr_, bytes_);
    }
    if (bound_) d.cuMulticastUnbind(mc_handle_, dev, 0, bytes_);
    if (uc_ptr_) {
      d.cuMemUnmap(uc_ptr_, bytes_);
      d.cuMemAddressFree(uc_ptr_, bytes_);
    }
    if (uc_handle_) d.cuMemRelease(uc_handle_);
    if (mc_handle_) d.cuMemRelease(mc_handle_);
  } catch (...) {
  }
}

int Multicast::create_and_export() {
  Driver& d = driver();
  CUmulticastObjectProp mp;
  memset(&mp, 0, sizeof(mp));
  mp.numDevices = unsigned(ranks_);
  mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  mp.size = prop_size_;
  CUmemGenericAllocationHandle h;
  ck(d.cuMulticastCreate(&h, &mp), "cuMulticastCreate");
  mc_handle_ = h;
  int fd = -1;
  ck(d.cuMemExportToShareableHandle(&fd, h, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0),
     "cuMemExportToShareableHandle(multicast)");
  return fd;
}

void Multicast::import_handle(int fd) {
  CUmemGenericAllocationHandle h;
  ck(driver().cuMemImportFromShareableHandle(&h, reinterpret_cast<void*>(static_cast<uintptr_t>(fd)),
                                             CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR),
     "cuMemImportFromShareableHandle(multicast)");
  mc_handle_ = h;
}

void Multicast::add_device() {
  Driver& d = driver();
  CUdevice dev;
  ck(d.cuDeviceGet(&dev, device_), "cuDeviceGet");
  ck(d.cuMulticastAddDevice(mc_handle_, dev), "cuMulticastAddDevice");
}

void Multicast::bind_and_map() {
  Driver& d = driver();
  CUmemAllocationProp p = device_prop(device_);
  CUmemGenericAllocationHandle uh;
  ck(d.cuMemCreate(&uh, bytes_, &p, 0), "cuMemCreate(multicast backing)");
  uc_handle_ = uh;
  ck(d.cuMulticastBindMem(mc_handle_, 0, uh, 0, bytes_, 0), "cuMulticastBindMem");
  bound_ = true;
  CUdeviceptr uva, mva;
  ck(d.cuMemAddressReserve(&uva, bytes_, gran_, 0, 0), "cuMemAddressReserve(uc)");
  uc_ptr_ = uva;
  map_rw(uva, bytes_, uh, device_);
  ck(d.cuMemAddressReserve(&mva, bytes_, gran_, 0, 0), "cuMemAddressReserve(mc)");
  mc_ptr_ = mva;
  map_rw(mva, bytes_, mc_handle_, device_);
}

}  // namespace sn
