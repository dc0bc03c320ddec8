// ckpt.cpp - checkpoint file helpers (see ckpt.h).
#include "ckpt.h"
#include <cstring>

namespace snnb {

namespace {
constexpr uint32_t NATIVE_MAGIC = 0x4E424E53u;  // "SNBN"
constexpr uint32_t NATIVE_VERSION = 1u;
constexpr size_t NAME_BYTES = 24;
constexpr size_t CHUNK = (size_t)64 << 20;
}  // namespace

BinFile::BinFile(const char* path, bool write) : path_(path ? path : "") {
    SNN_REQUIRE(path && *path, SNN_ERR_ARG, "empty checkpoint path");
    f_ = fopen(path, write ? "wb" : "rb");
    SNN_REQUIRE(f_, SNN_ERR_IO, std::string("cannot open ") + path_);
    if (!write) {
        fseeko(f_, 0, SEEK_END);
        size_ = (long long)ftello(f_);
        fseeko(f_, 0, SEEK_SET);
    }
}

BinFile::~BinFile() {
    if (f_) fclose(f_);
}

void BinFile::put(const void* p, size_t n) {
    SNN_REQUIRE(f_ && fwrite(p, 1, n, f_) == n, SNN_ERR_IO, "write failed: " + path_);
}

void BinFile::get(void* p, size_t n) {
    SNN_REQUIRE(f_ && fread(p, 1, n, f_) == n, SNN_ERR_IO, "truncated file: " + path_);
}

void BinFile::put_dev(const void* dev, size_t n, cudaStream_t st) {
    std::vector<char> buf(std::min(n, CHUNK));
    for (size_t off = 0; off < n; off += CHUNK) {
        const size_t m = std::min(CHUNK, n - off);
        SNN_CUDA(cudaMemcpyAsync(buf.data(), (const char*)dev + off, m, cudaMemcpyDeviceToHost, st));
        SNN_CUDA(cudaStreamSynchronize(st));
        put(buf.data(), m);
    }
}

void BinFile::get_dev(void* dev, size_t n, cudaStream_t st) {
    std::vector<char> buf(std::min(n, CHUNK));
    for (size_t off = 0; off < n; off += CHUNK) {
        const size_t m = std::min(CHUNK, n - off);
        get(buf.data(), m);
        SNN_CUDA(cudaMemcpyAsync((char*)dev + off, buf.data(), m, cudaMemcpyHostToDevice, st));
        SNN_CUDA(cudaStreamSynchronize(st));
    }
}

long long BinFile::tell() const { return f_ ? (long long)ftello(f_) : -1; }

void BinFile::seek(long long off) {
    SNN_REQUIRE(f_ && off >= 0 && off <= size_ && fseeko(f_, (off_t)off, SEEK_SET) == 0, SNN_ERR_IO,
                "seek failed: " + path_);
}

void BinFile::close() {
    if (!f_) return;
    const int rc = fclose(f_);
    f_ = nullptr;
    SNN_REQUIRE(rc == 0, SNN_ERR_IO, "close failed: " + path_);
}

void save_native(const char* path, int32_t model, const void* blob, uint32_t blob_bytes,
                 const std::vector<DevSection>& secs, cudaStream_t st) {
    SNN_CUDA(cudaStreamSynchronize(st));
    BinFile f(path, true);
    f.put_v(NATIVE_MAGIC);
    f.put_v(NATIVE_VERSION);
    f.put_v(model);
    f.put_v(blob_bytes);
    f.put(blob, blob_bytes);
    f.put_v((uint32_t)secs.size());
    for (const auto& s : secs) {
        char name[NAME_BYTES] = {0};
        strncpy(name, s.name, NAME_BYTES - 1);
        f.put(name, NAME_BYTES);
        f.put_v((uint64_t)s.bytes);
        if (s.bytes) f.put_dev(s.dev, s.bytes, st);
    }
    f.close();
}

void load_native(const char* path, int32_t model, void* blob, uint32_t blob_bytes,
                 const std::vector<DevSection>& secs, cudaStream_t st,
                 const std::function<void(const void*)>& check) {
    SNN_CUDA(cudaStreamSynchronize(st));
    BinFile f(path, false);
    long long expect = 4 * 4 + (long long)blob_bytes + 4;
    for (const auto& s : secs) expect += (long long)NAME_BYTES + 8 + (long long)s.bytes;
    SNN_REQUIRE(f.size() >= 16, SNN_ERR_IO, "truncated checkpoint");
    SNN_REQUIRE(f.get_v<uint32_t>() == NATIVE_MAGIC, SNN_ERR_IO, "not a native checkpoint (bad magic)");
    SNN_REQUIRE(f.get_v<uint32_t>() == NATIVE_VERSION, SNN_ERR_IO, "unsupported native checkpoint version");
    SNN_REQUIRE(f.get_v<int32_t>() == model, SNN_ERR_IO, "checkpoint of another model");
    SNN_REQUIRE(f.get_v<uint32_t>() == blob_bytes, SNN_ERR_IO, "checkpoint header size differs");
    SNN_REQUIRE(f.size() == expect, SNN_ERR_IO,
                "checkpoint size differs from this network's state (truncated, or another network)");
    std::vector<char> hb(blob_bytes);
    f.get(hb.data(), blob_bytes);
    SNN_REQUIRE(f.get_v<uint32_t>() == (uint32_t)secs.size(), SNN_ERR_IO, "checkpoint section count differs");
    // every section header is checked before anything reaches the device
    const long long first = f.tell();
    for (const auto& s : secs) {
        char name[NAME_BYTES];
        f.get(name, NAME_BYTES);
        const uint64_t nb = f.get_v<uint64_t>();
        SNN_REQUIRE(strncmp(name, s.name, NAME_BYTES) == 0 && nb == (uint64_t)s.bytes, SNN_ERR_IO,
                    std::string("checkpoint section differs at ") + s.name);
        if (s.validate) {
            std::vector<char> buf(std::min((size_t)nb, CHUNK));
            for (size_t off = 0; off < nb; off += CHUNK) {
                const size_t m = std::min(CHUNK, (size_t)nb - off);
                f.get(buf.data(), m);
                s.validate(buf.data(), m, off);
            }
        } else {
            f.seek(f.tell() + (long long)nb);
        }
    }
    if (check) check(hb.data());
    f.seek(first);
    for (const auto& s : secs) {
        f.seek(f.tell() + (long long)NAME_BYTES + 8);
        if (s.bytes) f.get_dev(s.dev, s.bytes, st);
    }
    memcpy(blob, hb.data(), blob_bytes);
}

}  // namespace snnb
