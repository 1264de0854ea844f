// Bundle file reader: maps a saved ProgramBundle (the .npz that
// llm_accelerator_b200/bundle.py ProgramBundle.save writes: uncompressed zip
// entries prefill.npy, decode.npy, shared.npy and meta.npy, each a 1-D uint8
// array) into memory and returns pointers into the mapping, so the
// instruction streams and the shared weight image reach their consumer (a
// host-to-device copy, a hash) without an intermediate copy.  The format
// stands in for the reference's in-memory ProgramBundle
// (software/taccel/assembler/assembler.py:163-548), which it persists.
//
// Zip: the end-of-central-directory record (zip64 form when present), the
// central directory's entries (zip64 extra field for sizes and offsets), each
// entry's local header; only stored (method 0) entries.  .npy: magic, format
// version 1-3, header dict with descr '|u1', no Fortran order, a 1-D shape.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdint>
#include <cstring>
#include <string>

#include "../../include/taccel_b200.h"

namespace {

struct Mapping {
  const uint8_t* base = nullptr;
  uint64_t size = 0;
};

uint16_t rd16(const uint8_t* p) { return uint16_t(p[0] | (p[1] << 8)); }
uint32_t rd32(const uint8_t* p) { return uint32_t(rd16(p)) | (uint32_t(rd16(p + 2)) << 16); }
uint64_t rd64(const uint8_t* p) { return uint64_t(rd32(p)) | (uint64_t(rd32(p + 4)) << 32); }

// Payload of a .npy file holding a 1-D uint8 array: *data, *len; false if
// the header is not that form or the payload does not fit in `avail` bytes.
bool npy_u8(const uint8_t* p, uint64_t avail, const uint8_t** data, uint64_t* len) {
  if (avail < 10 || std::memcmp(p, "\x93NUMPY", 6) != 0) return false;
  const int major = p[6];
  uint64_t hl = 0, off = 0;
  if (major == 1) {
    hl = rd16(p + 8);
    off = 10;
  } else if (major == 2 || major == 3) {
    if (avail < 12) return false;
    hl = rd32(p + 8);
    off = 12;
  } else {
    return false;
  }
  if (off + hl > avail) return false;
  const std::string h(reinterpret_cast<const char*>(p + off), hl);
  if (h.find("'descr': '|u1'") == std::string::npos && h.find("'descr': '<u1'") == std::string::npos)
    return false;
  if (h.find("'fortran_order': False") == std::string::npos) return false;
  const size_t s = h.find("'shape': (");
  if (s == std::string::npos) return false;
  size_t i = s + 10;
  uint64_t n = 0;
  bool digits = false;
  while (i < h.size() && h[i] >= '0' && h[i] <= '9') {
    n = n * 10 + uint64_t(h[i] - '0');
    digits = true;
    ++i;
  }
  // exactly one dimension: "(n,)" ; "(0,)" allowed
  if (!digits || i + 1 >= h.size() || h[i] != ',' || h[i + 1] != ')') return false;
  if (n > avail - off - hl) return false;
  *data = p + off + hl;
  *len = n;
  return true;
}

// True when [at, at + len) lies inside [0, n); written so that no sum wraps.
inline bool fits(uint64_t at, uint64_t len, uint64_t n) { return at <= n && len <= n - at; }

// Finds the stored entry `name`; its payload bounds in *off, *len.
int zip_entry(const Mapping& m, const char* name, uint64_t* off, uint64_t* len) {
  const uint8_t* b = m.base;
  const uint64_t n = m.size;
  if (n < 22) return TAC_E_ARGUMENT;
  // end of central directory: last occurrence of its signature within the final 64 KiB + 22 bytes
  int64_t eocd = -1;
  const uint64_t lo = n > 65557 ? n - 65557 : 0;
  for (uint64_t i = n - 22 + 1; i-- > lo;)
    if (rd32(b + i) == 0x06054b50u) {
      eocd = int64_t(i);
      break;
    }
  if (eocd < 0) return TAC_E_ARGUMENT;
  uint64_t cd_off = rd32(b + eocd + 16), cd_entries = rd16(b + eocd + 10);
  if (eocd >= 20 && rd32(b + eocd - 20) == 0x07064b50u) {   // zip64 locator
    const uint64_t z64 = rd64(b + eocd - 20 + 8);
    if (!fits(z64, 56, n) || rd32(b + z64) != 0x06064b50u) return TAC_E_ARGUMENT;
    cd_entries = rd64(b + z64 + 32);
    cd_off = rd64(b + z64 + 48);
  }
  uint64_t p = cd_off;
  const size_t want = std::strlen(name);
  for (uint64_t e = 0; e < cd_entries; ++e) {
    if (!fits(p, 46, n) || rd32(b + p) != 0x02014b50u) return TAC_E_ARGUMENT;
    const uint16_t method = rd16(b + p + 10);
    uint64_t csize = rd32(b + p + 20), usize = rd32(b + p + 24), lh = rd32(b + p + 42);
    const uint16_t nlen = rd16(b + p + 28), xlen = rd16(b + p + 30), clen = rd16(b + p + 32);
    if (!fits(p, 46 + uint64_t(nlen) + xlen + clen, n)) return TAC_E_ARGUMENT;
    const bool match = nlen == want && std::memcmp(b + p + 46, name, want) == 0;
    // zip64 extra field: the 0xFFFFFFFF fields in order usize, csize, local header offset
    for (uint64_t x = p + 46 + nlen; x + 4 <= p + 46 + nlen + xlen;) {
      const uint16_t id = rd16(b + x), sz = rd16(b + x + 2);
      if (x + 4 + sz > p + 46 + nlen + xlen) return TAC_E_ARGUMENT;
      if (id == 0x0001) {
        uint64_t q = x + 4;
        const uint64_t qend = x + 4 + sz;
        if (usize == 0xFFFFFFFFu && q + 8 <= qend) usize = rd64(b + q), q += 8;
        if (csize == 0xFFFFFFFFu && q + 8 <= qend) csize = rd64(b + q), q += 8;
        if (lh == 0xFFFFFFFFu && q + 8 <= qend) lh = rd64(b + q), q += 8;
      }
      x += 4 + sz;
    }
    if (match) {
      if (method != 0 || csize != usize) return TAC_E_UNSUPPORTED;   // compressed entry
      if (!fits(lh, 30, n) || rd32(b + lh) != 0x04034b50u) return TAC_E_ARGUMENT;
      const uint64_t data = lh + 30 + rd16(b + lh + 26) + rd16(b + lh + 28);
      if (data > n || csize > n - data) return TAC_E_ARGUMENT;
      *off = data;
      *len = csize;
      return TAC_OK;
    }
    p += 46 + uint64_t(nlen) + xlen + clen;
  }
  return TAC_E_ARGUMENT;   // entry missing
}

}  // namespace

extern "C" int tac_bundle_open(const char* path, tac_bundle_view* view, void** handle) {
  if (!path || !view || !handle) return TAC_E_ARGUMENT;
  *handle = nullptr;
  const int fd = ::open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) return TAC_E_ARGUMENT;
  struct stat st;
  if (::fstat(fd, &st) != 0 || st.st_size <= 0) {
    ::close(fd);
    return TAC_E_ARGUMENT;
  }
  void* base = ::mmap(nullptr, size_t(st.st_size), PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (base == MAP_FAILED) return TAC_E_ARGUMENT;
  Mapping* m = new Mapping{static_cast<const uint8_t*>(base), uint64_t(st.st_size)};
  const char* names[4] = {"prefill.npy", "decode.npy", "shared.npy", "meta.npy"};
  const uint8_t* ptrs[4] = {};
  uint64_t lens[4] = {};
  for (int i = 0; i < 4; ++i) {
    uint64_t off = 0, len = 0;
    int rc = zip_entry(*m, names[i], &off, &len);
    if (rc == TAC_OK && !npy_u8(m->base + off, len, &ptrs[i], &lens[i])) rc = TAC_E_ARGUMENT;
    if (rc != TAC_OK) {
      ::munmap(const_cast<uint8_t*>(m->base), size_t(m->size));
      delete m;
      return rc;
    }
  }
  view->prefill = ptrs[0];
  view->prefill_len = lens[0];
  view->decode = ptrs[1];
  view->decode_len = lens[1];
  view->shared = ptrs[2];
  view->shared_len = lens[2];
  view->meta_json = reinterpret_cast<const char*>(ptrs[3]);
  view->meta_len = lens[3];
  *handle = m;
  return TAC_OK;
}

extern "C" int tac_bundle_close(void* handle) {
  if (!handle) return TAC_E_ARGUMENT;
  Mapping* m = static_cast<Mapping*>(handle);
  ::munmap(const_cast<uint8_t*>(m->base), size_t(m->size));
  delete m;
  return TAC_OK;
}
