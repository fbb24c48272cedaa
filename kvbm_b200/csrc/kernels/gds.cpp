// GPUDirect Storage (cuFile) I/O between device memory and a G3 block file:
// G1 <-> G3 without the pinned-host bounce of the two-hop path. libcufile is
// opened at run time (dlopen), so the library loads, and the two-hop path
// stays available, on hosts without it. Without the nvidia-fs driver cuFile
// runs in its compatibility mode (POSIX I/O through its own staging buffers);
// the calls and their results are the same.
//
// Parity: crates/kvbm-physical/src/transfer/capabilities.rs (allow_gds),
// strategy.rs (device <-> disk direct when GDS is allowed); the reference
// reaches GDS through NIXL's GDS / GDS_MT backends.
#include <cuda.h>
#include <cufile.h>
#include <dlfcn.h>
#include <fcntl.h>
#include <unistd.h>

#include <cerrno>
#include <cstdint>
#include <cstring>
#include <mutex>

namespace {

struct CuFileApi {
  decltype(&cuFileDriverOpen) driver_open = nullptr;
  decltype(&cuFileHandleRegister) handle_register = nullptr;
  decltype(&cuFileHandleDeregister) handle_deregister = nullptr;
  decltype(&cuFileBufRegister) buf_register = nullptr;
  decltype(&cuFileBufDeregister) buf_deregister = nullptr;
  decltype(&cuFileRead) read = nullptr;
  decltype(&cuFileWrite) write = nullptr;
  int status = -1;  // 0: usable; 1: no libcufile; 2: missing symbol; 1000 + CUfileOpError: driver open failed
};

CuFileApi g_api;
std::once_flag g_once;

template <typename F>
bool sym(void* lib, const char* name, F& out) {
  out = reinterpret_cast<F>(dlsym(lib, name));
  return out != nullptr;
}

void load_api() {
  void* lib = dlopen("libcufile.so.0", RTLD_NOW | RTLD_LOCAL);
  if (!lib) lib = dlopen("libcufile.so", RTLD_NOW | RTLD_LOCAL);
  if (!lib) {
    g_api.status = 1;
    return;
  }
  bool ok = sym(lib, "cuFileDriverOpen", g_api.driver_open) &&
            sym(lib, "cuFileHandleRegister", g_api.handle_register) &&
            sym(lib, "cuFileHandleDeregister", g_api.handle_deregister) &&
            sym(lib, "cuFileBufRegister", g_api.buf_register) &&
            sym(lib, "cuFileBufDeregister", g_api.buf_deregister) && sym(lib, "cuFileRead", g_api.read) &&
            sym(lib, "cuFileWrite", g_api.write);
  if (!ok) {
    g_api.status = 2;
    return;
  }
  const CUfileError_t e = g_api.driver_open();
  g_api.status = e.err == CU_FILE_SUCCESS ? 0 : 1000 + static_cast<int>(e.err);
}

struct GdsFile {
  int fd;
  CUfileHandle_t fh;
};

}  // namespace

// 0 when cuFile is usable in this process, else the reason (see CuFileApi::status).
extern "C" int kvbm_gds_status() {
  std::call_once(g_once, load_api);
  return g_api.status;
}

namespace {
// Register `fd` (owned by the new handle) with cuFile.
int open_fd(int fd, void** out) {
  CUfileDescr_t d;
  std::memset(&d, 0, sizeof(d));
  d.handle.fd = fd;
  d.type = CU_FILE_HANDLE_TYPE_OPAQUE_FD;
  CUfileHandle_t fh = nullptr;
  const CUfileError_t e = g_api.handle_register(&fh, &d);
  if (e.err != CU_FILE_SUCCESS) {
    close(fd);
    return 1000 + static_cast<int>(e.err);
  }
  *out = new GdsFile{fd, fh};
  return 0;
}
}  // namespace

// Open `path` (which must exist) for cuFile I/O; O_DIRECT when `direct` and the
// file system allows it. Returns 0 and a handle, or an errno / cuFile code.
extern "C" int kvbm_gds_open(const char* path, int direct, void** out) {
  if (!path || !out) return EINVAL;
  if (int s = kvbm_gds_status()) return s;
  int fd = -1;
  if (direct) fd = open(path, O_RDWR | O_DIRECT);
  if (fd < 0) fd = open(path, O_RDWR);
  if (fd < 0) return errno;
  return open_fd(fd, out);
}

// The same for an already open descriptor (duplicated: the caller keeps its own),
// e.g. a disk pool whose file was unlinked after opening.
extern "C" int kvbm_gds_open_fd(int fd, void** out) {
  if (fd < 0 || !out) return EINVAL;
  if (int s = kvbm_gds_status()) return s;
  const int dup_fd = dup(fd);
  if (dup_fd < 0) return errno;
  return open_fd(dup_fd, out);
}

extern "C" int kvbm_gds_close(void* h) {
  if (!h) return 0;
  auto* f = static_cast<GdsFile*>(h);
  g_api.handle_deregister(f->fh);
  close(f->fd);
  delete f;
  return 0;
}

// Optional: pin a device range for cuFile (avoids its internal staging copies).
extern "C" int kvbm_gds_register_buffer(const void* dev, size_t bytes) {
  if (int s = kvbm_gds_status()) return s;
  const CUfileError_t e = g_api.buf_register(dev, bytes, 0);
  return e.err == CU_FILE_SUCCESS ? 0 : 1000 + static_cast<int>(e.err);
}

extern "C" int kvbm_gds_deregister_buffer(const void* dev) {
  if (int s = kvbm_gds_status()) return s;
  const CUfileError_t e = g_api.buf_deregister(dev);
  return e.err == CU_FILE_SUCCESS ? 0 : 1000 + static_cast<int>(e.err);
}

// Move `bytes` between device memory (dev_base + dev_offset) and the file at
// `file_offset`; `write` != 0: device -> file. Synchronous; partial transfers
// are continued. Returns the bytes moved, or a negative errno or negative cuFile error code.
extern "C" int64_t kvbm_gds_io(void* h, int write, void* dev_base, int64_t dev_offset, int64_t file_offset,
                               int64_t bytes) {
  if (!h || !dev_base || bytes < 0) return -EINVAL;
  auto* f = static_cast<GdsFile*>(h);
  int64_t done = 0;
  while (done < bytes) {
    const ssize_t n = write ? g_api.write(f->fh, dev_base, static_cast<size_t>(bytes - done), file_offset + done,
                                          dev_offset + done)
                            : g_api.read(f->fh, dev_base, static_cast<size_t>(bytes - done), file_offset + done,
                                         dev_offset + done);
    if (n < 0) return n == -1 ? -errno : static_cast<int64_t>(n);
    if (n == 0) return write ? -EIO : done;  // a read past the end of the file stops early
    done += n;
  }
  return done;
}
