// ckpt.h - checkpoint file helpers shared by the engines (host side).
//
// BinFile: binary file with checked writes / exact reads (SNN_ERR_IO on any
// failure, "truncated" on a short read) and chunked device <-> file copies.
//
// Native full-state format (SNN_FMT_NATIVE), for bit-exact resume:
//   u32 magic 0x4E424E53 ("SNBN"), u32 version 1, i32 model,
//   u32 blob bytes, blob (the engine's host-side state),
//   u32 section count, then per section: char name[24], u64 bytes, data.
// A loader checks magic, version, model, blob size and every section's name
// and size against what the engine expects, and the file's total size,
// before it writes anything to the device.
#pragma once
#include <cstdio>
#include <functional>
#include <string>
#include <vector>
#include "common.h"

namespace snnb {

class BinFile {
public:
    BinFile(const char* path, bool write);
    ~BinFile();
    BinFile(const BinFile&) = delete;
    BinFile& operator=(const BinFile&) = delete;
    void put(const void* p, size_t n);
    void get(void* p, size_t n);
    template <typename T> void put_v(const T& v) { put(&v, sizeof(T)); }
    template <typename T> T get_v() { T v; get(&v, sizeof(T)); return v; }
    // device memory <-> file in bounded host chunks (synchronises `st`)
    void put_dev(const void* dev, size_t n, cudaStream_t st);
    void get_dev(void* dev, size_t n, cudaStream_t st);
    long long size() const { return size_; }  // file size when opened for reading
    long long tell() const;
    void seek(long long off);                   // absolute, within the file (reading)
    void close();                               // flush + close, checked

private:
    FILE* f_ = nullptr;
    std::string path_;
    long long size_ = 0;
};

struct DevSection {
    const char* name;
    void* dev;
    size_t bytes;
    // optional: sees the file's data of the section, in chunks (offset in
    // bytes from its start), before anything reaches the device; throws to
    // refuse the file
    std::function<void(const char*, size_t, size_t)> validate = nullptr;
};

void save_native(const char* path, int32_t model, const void* blob, uint32_t blob_bytes,
                 const std::vector<DevSection>& secs, cudaStream_t st);
// `check` (optional) sees the file's blob before anything reaches the device
// and throws to refuse it
void load_native(const char* path, int32_t model, void* blob, uint32_t blob_bytes,
                 const std::vector<DevSection>& secs, cudaStream_t st,
                 const std::function<void(const void*)>& check = nullptr);

}  // namespace snnb
