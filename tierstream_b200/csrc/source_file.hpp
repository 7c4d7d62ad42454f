// A descriptor source file opened for reading: unbuffered (O_DIRECT) when asked and allowed, else buffered. Reads of
// any offset and size; unbuffered reads go through an aligned bounce buffer of the file's alignment.
#pragma once

#include <cstdint>
#include <string>

namespace tsb {

class SourceFile {
 public:
  SourceFile(const std::string& path, uint64_t align, bool direct);
  ~SourceFile();
  SourceFile(const SourceFile&) = delete;
  SourceFile& operator=(const SourceFile&) = delete;
  // Reads exactly `bytes` at `offset` into dst (throws SS_E_IO on a short read or an error). Thread-safe.
  void read(void* dst, uint64_t offset, uint64_t bytes) const;
  bool direct() const { return direct_; }
  uint64_t size() const { return size_; }
  const std::string& path() const { return path_; }

 private:
  std::string path_;
  int fd_ = -1, fd_buffered_ = -1;
  bool direct_ = false;
  uint64_t align_ = 4096, size_ = 0;
};

}  // namespace tsb
