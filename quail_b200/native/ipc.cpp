// Worker IPC for the per-GPU worker processes: Unix-domain sockets carrying
// length-prefixed frames, process spawn / liveness / kill, and shared-memory
// tables in /dev/shm.
//
// Frame format (the reference's, crates/quail/src/workers.rs:43-60): an
// 8-byte little-endian payload length, then the payload (JSON text or an
// Arrow IPC stream). A reader refuses a length above its limit before
// allocating, so a corrupt or hostile peer cannot make it allocate
// unbounded memory. Every blocking call takes a timeout.
//
// Shared tables (crates/quail/src/shared.rs:45-108): the payload is written
// once into a /dev/shm file that every worker maps read-only; the file name
// is unlinked by the owner once all readers have mapped it.
#include <errno.h>
#include <fcntl.h>
#include <poll.h>
#include <signal.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/socket.h>
#include <sys/stat.h>
#include <sys/types.h>
#include <sys/un.h>
#include <sys/wait.h>
#include <time.h>
#include <unistd.h>

#include <chrono>
#include <string>
#include <vector>

#include "ipc.h"

extern char** environ;

namespace qbn {

namespace {

long long now_ms() {
  return std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now().time_since_epoch())
      .count();
}

[[noreturn]] void sys_fail(const std::string& what) { throw IpcError(what + ": " + strerror(errno)); }

// wait until fd is readable/writable or the deadline passes
void wait_fd(int fd, short events, long long deadline_ms, const char* what) {
  while (true) {
    long long left = deadline_ms < 0 ? -1 : deadline_ms - now_ms();
    if (deadline_ms >= 0 && left <= 0) throw IpcTimeout(std::string("timed out waiting to ") + what);
    struct pollfd p = {fd, events, 0};
    int r = poll(&p, 1, left < 0 ? -1 : (int)std::min<long long>(left, 1 << 30));
    if (r < 0) {
      if (errno == EINTR) continue;
      sys_fail("poll");
    }
    if (r == 0) continue;
    if (p.revents & (POLLERR | POLLNVAL)) throw IpcError(std::string("socket error while waiting to ") + what);
    if (p.revents & (events | POLLHUP)) return;
  }
}

void write_all(int fd, const char* data, size_t n, long long deadline) {
  size_t off = 0;
  while (off < n) {
    wait_fd(fd, POLLOUT, deadline, "send");
    ssize_t w = ::send(fd, data + off, n - off, MSG_NOSIGNAL);
    if (w < 0) {
      if (errno == EINTR || errno == EAGAIN) continue;
      sys_fail("send");
    }
    off += (size_t)w;
  }
}

void read_all(int fd, char* data, size_t n, long long deadline) {
  size_t off = 0;
  while (off < n) {
    wait_fd(fd, POLLIN, deadline, "receive");
    ssize_t r = ::recv(fd, data + off, n - off, 0);
    if (r < 0) {
      if (errno == EINTR || errno == EAGAIN) continue;
      sys_fail("recv");
    }
    if (r == 0) throw IpcClosed("peer closed the connection");
    off += (size_t)r;
  }
}

sockaddr_un unix_addr(const std::string& path) {
  sockaddr_un a{};
  a.sun_family = AF_UNIX;
  if (path.size() >= sizeof(a.sun_path)) throw IpcError("socket path too long: " + path);
  strncpy(a.sun_path, path.c_str(), sizeof(a.sun_path) - 1);
  return a;
}

}  // namespace

// ------------------------------------------------------------ frames
void send_frame(int fd, const std::string& payload, int timeout_ms) {
  const long long deadline = timeout_ms < 0 ? -1 : now_ms() + timeout_ms;
  unsigned char hdr[8];
  uint64_t n = payload.size();
  for (int i = 0; i < 8; ++i) hdr[i] = (unsigned char)((n >> (8 * i)) & 0xff);
  write_all(fd, reinterpret_cast<const char*>(hdr), 8, deadline);
  write_all(fd, payload.data(), payload.size(), deadline);
}

std::string recv_frame(int fd, uint64_t max_bytes, int timeout_ms) {
  const long long deadline = timeout_ms < 0 ? -1 : now_ms() + timeout_ms;
  unsigned char hdr[8];
  read_all(fd, reinterpret_cast<char*>(hdr), 8, deadline);
  uint64_t n = 0;
  for (int i = 0; i < 8; ++i) n |= (uint64_t)hdr[i] << (8 * i);
  if (n > max_bytes)
    throw IpcError("frame of " + std::to_string(n) + " bytes exceeds the limit of " + std::to_string(max_bytes));
  std::string out(n, '\0');
  read_all(fd, out.data(), n, deadline);
  return out;
}

// ------------------------------------------------------------ sockets
int listen_unix(const std::string& path) {
  ::unlink(path.c_str());
  int fd = ::socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
  if (fd < 0) sys_fail("socket");
  sockaddr_un a = unix_addr(path);
  if (::bind(fd, reinterpret_cast<sockaddr*>(&a), sizeof a) < 0) {
    ::close(fd);
    sys_fail("bind " + path);
  }
  if (::listen(fd, 64) < 0) {
    ::close(fd);
    sys_fail("listen");
  }
  return fd;
}

int accept_unix(int listen_fd, int timeout_ms) {
  wait_fd(listen_fd, POLLIN, timeout_ms < 0 ? -1 : now_ms() + timeout_ms, "accept a worker");
  int fd = ::accept4(listen_fd, nullptr, nullptr, SOCK_CLOEXEC);
  if (fd < 0) sys_fail("accept");
  return fd;
}

int connect_unix(const std::string& path, int patience_ms) {
  const long long deadline = now_ms() + patience_ms;
  while (true) {
    int fd = ::socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
    if (fd < 0) sys_fail("socket");
    sockaddr_un a = unix_addr(path);
    if (::connect(fd, reinterpret_cast<sockaddr*>(&a), sizeof a) == 0) return fd;
    const int e = errno;
    ::close(fd);
    if (e != ENOENT && e != ECONNREFUSED) {
      errno = e;
      sys_fail("connect " + path);
    }
    if (now_ms() > deadline) throw IpcTimeout("no listener at " + path + " within the patience");
    struct timespec ts = {0, 20 * 1000 * 1000};
    nanosleep(&ts, nullptr);
  }
}

void close_fd(int fd) {
  if (fd >= 0) ::close(fd);
}

// ------------------------------------------------------------ processes
int spawn(const std::vector<std::string>& argv, const std::vector<std::string>& env_overrides) {
  if (argv.empty()) throw IpcError("spawn: empty argv");
  std::vector<std::string> env;
  for (char** e = environ; *e; ++e) {
    std::string kv(*e);
    const std::string key = kv.substr(0, kv.find('='));
    bool replaced = false;
    for (const auto& o : env_overrides)
      if (o.substr(0, o.find('=')) == key) replaced = true;
    if (!replaced) env.push_back(kv);
  }
  for (const auto& o : env_overrides) env.push_back(o);
  std::vector<char*> cargv, cenv;
  for (const auto& a : argv) cargv.push_back(const_cast<char*>(a.c_str()));
  cargv.push_back(nullptr);
  for (const auto& e : env) cenv.push_back(const_cast<char*>(e.c_str()));
  cenv.push_back(nullptr);
  pid_t pid = ::fork();
  if (pid < 0) sys_fail("fork");
  if (pid == 0) {
    ::execve(cargv[0], cargv.data(), cenv.data());
    _exit(127);
  }
  return (int)pid;
}

// -1: still running; otherwise the exit status (128 + signal when killed)
int poll_exit(int pid) {
  int status = 0;
  pid_t r = ::waitpid(pid, &status, WNOHANG);
  if (r == 0) return -1;
  if (r < 0) return errno == ECHILD ? 0 : -2;
  if (WIFEXITED(status)) return WEXITSTATUS(status);
  if (WIFSIGNALED(status)) return 128 + WTERMSIG(status);
  return 0;
}

void kill_pid(int pid, int sig) {
  if (pid > 0) ::kill(pid, sig);
}

// ------------------------------------------------------------ shared tables
std::string shm_write(const std::string& name, const std::string& bytes) {
  std::string path = "/dev/shm/" + name;
  int fd = ::open(path.c_str(), O_CREAT | O_TRUNC | O_RDWR | O_CLOEXEC, 0600);
  if (fd < 0) sys_fail("open " + path);
  size_t off = 0;
  while (off < bytes.size()) {
    ssize_t w = ::write(fd, bytes.data() + off, bytes.size() - off);
    if (w < 0) {
      if (errno == EINTR) continue;
      ::close(fd);
      sys_fail("write " + path);
    }
    off += (size_t)w;
  }
  ::close(fd);
  return path;
}

MappedFile::MappedFile(const std::string& path) {
  int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
  if (fd < 0) sys_fail("open " + path);
  struct stat st;
  if (::fstat(fd, &st) < 0) {
    ::close(fd);
    sys_fail("stat " + path);
  }
  size_ = (size_t)st.st_size;
  if (size_) {
    data_ = ::mmap(nullptr, size_, PROT_READ, MAP_SHARED, fd, 0);
    if (data_ == MAP_FAILED) {
      ::close(fd);
      sys_fail("mmap " + path);
    }
  }
  ::close(fd);
}

MappedFile::~MappedFile() {
  if (data_ && data_ != MAP_FAILED) ::munmap(data_, size_);
}

void unlink_path(const std::string& path) { ::unlink(path.c_str()); }

}  // namespace qbn
