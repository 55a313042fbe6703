#include "model_file.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <limits>
#include <stdexcept>

#include "status_error.h"

namespace dav2 {
namespace {

#pragma pack(push, 1)
struct Header {
    char magic[8];
    std::uint32_t version, endian, encoder, tensor_count;
    std::uint64_t directory_offset, directory_bytes, data_offset, file_bytes, metadata_offset;
};
struct Record {
    char name[112];
    std::uint32_t dtype, rank;
    std::uint64_t dims[4];
    std::uint64_t data_offset, data_bytes, element_count;
    std::uint32_t crc32, flags;
    std::uint64_t reserved;
};
struct Metadata {
    char magic[8];
    std::uint32_t version, bytes, model_format_version, encoder, flags, max_depth_bits;
    std::uint8_t canonical_sha256[32];
    char converter[64];
};
#pragma pack(pop)
static_assert(sizeof(Header) == 64, "header is 64 bytes");
static_assert(sizeof(Record) == 192, "record is 192 bytes");
static_assert(sizeof(Metadata) == 128, "metadata is 128 bytes");

bool in_bounds(std::uint64_t offset, std::uint64_t bytes, std::uint64_t limit) {
    return offset <= limit && bytes <= limit - offset;
}

}  // namespace

std::uint32_t crc32(const void* data, std::size_t bytes) {
    static std::uint32_t table[256];
    static const bool ready = [] {
        for (std::uint32_t n = 0; n < 256; ++n) {
            std::uint32_t c = n;
            for (int k = 0; k < 8; ++k) c = (c & 1u) ? 0xedb88320u ^ (c >> 1) : c >> 1;
            table[n] = c;
        }
        return true;
    }();
    (void)ready;
    const auto* p = static_cast<const unsigned char*>(data);
    std::uint32_t crc = 0xffffffffu;
    for (std::size_t i = 0; i < bytes; ++i) crc = table[(crc ^ p[i]) & 0xffu] ^ (crc >> 8);
    return crc ^ 0xffffffffu;
}

ModelFile::ModelFile(const std::string& path, dav2_encoder expected) {
    if (path.empty()) throw std::invalid_argument("model path is empty");
    try {
        fd_ = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
        if (fd_ < 0) throw_model_io("failed to open model file");
        struct stat st {};
        if (fstat(fd_, &st) != 0 || st.st_size < 0) throw_model_io("failed to query model file size");
        size_ = static_cast<std::uint64_t>(st.st_size);
        if (size_ < sizeof(Header)) throw_model_format("model file is truncated or too large");
        void* m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
        if (m == MAP_FAILED) throw_model_io("failed to map model file");
        view_ = static_cast<const unsigned char*>(m);

        Header h;
        std::memcpy(&h, view_, sizeof h);
        if (std::memcmp(h.magic, "DAV2MOD\0", 8) != 0 || h.version != 1 || h.endian != 0x01020304u)
            throw_model_format("invalid DAV2 model header");
        if (h.encoder != static_cast<std::uint32_t>(expected))
            throw_model_format("model encoder does not match create options");
        if (h.tensor_count == 0 || h.tensor_count > 2048 || h.file_bytes != size_)
            throw_model_format("invalid DAV2 model bounds");
        if (h.directory_bytes != std::uint64_t(h.tensor_count) * sizeof(Record) ||
            !in_bounds(h.directory_offset, h.directory_bytes, size_) || h.data_offset % 64 != 0 ||
            h.data_offset < h.directory_offset + h.directory_bytes || h.data_offset > size_)
            throw_model_format("invalid DAV2 tensor directory");
        if (h.metadata_offset != 0) {
            if (h.metadata_offset != h.directory_offset + h.directory_bytes ||
                !in_bounds(h.metadata_offset, sizeof(Metadata), h.data_offset))
                throw_model_format("invalid DAV2 derivation metadata bounds");
            Metadata md;
            std::memcpy(&md, view_ + h.metadata_offset, sizeof md);
            if (std::memcmp(md.magic, "DAV2META", 8) != 0 || md.version != 1 || md.bytes != sizeof(Metadata) ||
                md.model_format_version != 1 || md.encoder != h.encoder || (md.flags & ~1u) != 0 ||
                std::memchr(md.converter, '\0', sizeof md.converter) == nullptr)
                throw_model_format("invalid DAV2 derivation metadata");
            const std::string converter(md.converter);
            if (md.flags & 1u) {
                float depth;
                std::memcpy(&depth, &md.max_depth_bits, sizeof depth);
                if (converter != "dav2-export-pytorch-metric-v1")
                    throw_model_format("invalid DAV2 metric converter identity");
                if (depth != 20.0f && depth != 80.0f) throw_model_format("invalid DAV2 metric maximum depth");
                metric_max_depth_ = depth;
            } else if (md.max_depth_bits != 0) {
                throw_model_format("invalid DAV2 relative derivation metadata");
            } else if (converter != "dav2-export-pytorch-v1") {
                throw_model_format("invalid DAV2 relative converter identity");
            }
        }
        tensors_.reserve(h.tensor_count);
        names_.reserve(h.tensor_count);
        for (std::uint32_t i = 0; i < h.tensor_count; ++i) {
            Record r;
            std::memcpy(&r, view_ + h.directory_offset + std::uint64_t(i) * sizeof(Record), sizeof r);
            const void* end = std::memchr(view_ + h.directory_offset + std::uint64_t(i) * sizeof(Record), '\0', 112);
            if (!end || r.name[0] == '\0' || r.dtype != 1 || r.rank == 0 || r.rank > 4 || r.flags != 0 ||
                r.reserved != 0 || r.data_offset < h.data_offset || r.data_offset % 64 != 0 ||
                !in_bounds(r.data_offset, r.data_bytes, size_))
                throw_model_format("invalid DAV2 tensor record");
            std::uint64_t elements = 1;
            for (std::uint32_t d = 0; d < 4; ++d) {
                if (d < r.rank) {
                    if (r.dims[d] == 0 || elements > std::numeric_limits<std::uint64_t>::max() / r.dims[d])
                        throw_model_format("invalid DAV2 tensor dimensions");
                    elements *= r.dims[d];
                } else if (r.dims[d] != 0) {
                    throw_model_format("invalid DAV2 unused dimension");
                }
            }
            if (elements != r.element_count || elements * 4 != r.data_bytes)
                throw_model_format("invalid DAV2 tensor byte count");
            const char* name = reinterpret_cast<const char*>(view_ + h.directory_offset + std::uint64_t(i) * sizeof(Record));
            std::string_view key(name, static_cast<const char*>(end) - name);
            TensorView tv;
            tv.data = reinterpret_cast<const float*>(view_ + r.data_offset);
            tv.dims = {r.dims[0], r.dims[1], r.dims[2], r.dims[3]};
            tv.rank = r.rank;
            tv.elements = r.element_count;
            tv.crc32 = r.crc32;
            if (!tensors_.emplace(key, tv).second) throw_model_format("duplicate DAV2 tensor name");
            names_.push_back(key);
        }
    } catch (...) {
        unmap();
        throw;
    }
}

ModelFile::~ModelFile() { unmap(); }

void ModelFile::unmap() noexcept {
    tensors_.clear();
    names_.clear();
    if (view_) munmap(const_cast<unsigned char*>(view_), size_);
    view_ = nullptr;
    if (fd_ >= 0) ::close(fd_);
    fd_ = -1;
}

const TensorView& ModelFile::tensor(std::string_view name) const {
    auto it = tensors_.find(name);
    if (it == tensors_.end()) throw_model_format("model is missing tensor: " + std::string(name));
    return it->second;
}

void ModelFile::verify_crc() const {
    for (const auto& [name, t] : tensors_)
        if (crc32(t.data, t.elements * 4) != t.crc32)
            throw_model_format("CRC-32 mismatch for tensor " + std::string(name));
}

}  // namespace dav2
