// Worker IPC declarations (see ipc.cpp).
#pragma once

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

namespace qbn {

struct IpcError : std::runtime_error {
  using std::runtime_error::runtime_error;
};
struct IpcTimeout : IpcError {
  using IpcError::IpcError;
};
struct IpcClosed : IpcError {
  using IpcError::IpcError;
};

void send_frame(int fd, const std::string& payload, int timeout_ms);
std::string recv_frame(int fd, uint64_t max_bytes, int timeout_ms);
int listen_unix(const std::string& path);
int accept_unix(int listen_fd, int timeout_ms);
int connect_unix(const std::string& path, int patience_ms);
void close_fd(int fd);
int spawn(const std::vector<std::string>& argv, const std::vector<std::string>& env_overrides);
int poll_exit(int pid);
void kill_pid(int pid, int sig);
std::string shm_write(const std::string& name, const std::string& bytes);
void unlink_path(const std::string& path);

class MappedFile {
 public:
  explicit MappedFile(const std::string& path);
  ~MappedFile();
  MappedFile(const MappedFile&) = delete;
  MappedFile& operator=(const MappedFile&) = delete;
  const void* data() const { return data_; }
  size_t size() const { return size_; }

 private:
  void* data_ = nullptr;
  size_t size_ = 0;
};

}  // namespace qbn
