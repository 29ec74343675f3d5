// Symmetric-memory bootstrap (see symm_mem.cpp).
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <string>
#include <vector>

namespace sn {

// Descriptor passing over abstract unix sockets (SCM_RIGHTS).
int fd_listen(const std::string& name);
void fd_serve(int listener, int fd, int clients, int timeout_ms);
int fd_fetch(const std::string& name, int timeout_ms);
void fd_close(int fd);

size_t vmm_granularity(int device);
int device_attribute(int device, int attr);
bool multicast_supported(int device);

// One rank's physical region, mapped locally, plus mappings of peers' regions.
class LocalRegion {
 public:
  LocalRegion(int device, size_t bytes, size_t align);
  ~LocalRegion();
  LocalRegion(const LocalRegion&) = delete;
  LocalRegion& operator=(const LocalRegion&) = delete;
  uint64_t ptr() const { return ptr_; }
  size_t bytes() const { return bytes_; }
  int export_fd() const;
  uint64_t map_peer(int fd, size_t bytes);

 private:
  struct PeerMap {
    uint64_t ptr;
    size_t bytes;
    unsigned long long handle;
  };
  int device_;
  size_t bytes_ = 0;
  uint64_t ptr_ = 0;
  unsigned long long handle_ = 0;
  std::vector<PeerMap> peers_;
};

// The NVLS multicast object and this rank's bound backing memory.
class Multicast {
 public:
  Multicast(int device, size_t bytes, int ranks);
  ~Multicast();
  Multicast(const Multicast&) = delete;
  Multicast& operator=(const Multicast&) = delete;
  int create_and_export();        // rank 0
  void import_handle(int fd);     // other ranks
  void add_device();              // every rank, before anyone binds
  void bind_and_map();            // every rank, after all devices joined
  uint64_t mc_ptr() const { return mc_ptr_; }
  uint64_t uc_ptr() const { return uc_ptr_; }
  size_t bytes() const { return bytes_; }

 private:
  int device_;
  int ranks_;
  size_t bytes_ = 0, gran_ = 0, prop_size_ = 0;
  unsigned long long mc_handle_ = 0, uc_handle_ = 0;
  uint64_t mc_ptr_ = 0, uc_ptr_ = 0;
  bool bound_ = false;
};

}  // namespace sn
