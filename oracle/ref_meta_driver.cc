// Test oracle driver: runs the REFERENCE's KVCacheMetadata and
// KVCacheMetadataShmRegion (tpu_sync/kv_cache/kv_cache_metadata.cc,
// kv_cache_metadata_shm.cc, compiled where they lie by oracle/build_ref.py)
// over a command script read from stdin, so tests can compare the product's
// table bytes, entries and error statuses with the reference's.
//
// Commands (one per line; strings are hex, "-" for empty):
//   region N              fresh zeroed 64-byte aligned buffer of N bytes
//   load PATH / save PATH  buffer <- / -> file
//   poke OFF HEX           overwrite buffer bytes (a torn or foreign table)
//   dump                   print the buffer as "bytes HEX"
//   format NB UID [OFF LEN]  KVCacheMetadata::Format on the buffer (or on
//   attach NB UID [OFF LEN]  its subspan [OFF, OFF+LEN)); "null" for OFF
//                            formats an empty span
//   set ID HASH SEQ / clear ID / entries
//   shm KEY NB UID         KVCacheMetadataShmRegion::AttachOrFormat
//   shm_reformat / shm_close
// Every command prints "ok", "ok warm=W", or "err CODE MESSAGE"; entries
// prints "entry ID HASH SEQ" lines and then "end".
//
// Test infrastructure only: nothing in the product links or runs this.

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <iostream>
#include <memory>
#include <optional>
#include <sstream>
#include <string>
#include <vector>

#include "tpu_sync/kv_cache/kv_cache_metadata.h"
#include "tpu_sync/kv_cache/kv_cache_metadata_shm.h"

using tpu_raiden::kv_cache::KVCacheMetadata;
using tpu_raiden::kv_cache::KVCacheMetadataShmRegion;

namespace {

std::string unhex(const std::string& h) {
  if (h == "-") return "";
  std::string out;
  for (size_t i = 0; i + 1 < h.size(); i += 2) out.push_back(char(std::stoi(h.substr(i, 2), nullptr, 16)));
  return out;
}

std::string hex(const std::string& s) {
  if (s.empty()) return "-";
  static const char* d = "0123456789abcdef";
  std::string out;
  for (unsigned char c : s) {
    out.push_back(d[c >> 4]);
    out.push_back(d[c & 15]);
  }
  return out;
}

void report(const absl::Status& s) {
  if (s.ok())
    std::cout << "ok\n";
  else
    std::cout << "err " << int(s.code()) << " " << s.message() << "\n";
}

}  // namespace

int main() {
  std::vector<uint8_t> raw;
  uint8_t* buf = nullptr;
  size_t buf_len = 0;
  std::optional<KVCacheMetadata> meta;
  std::unique_ptr<KVCacheMetadataShmRegion> shm;
  auto set_region = [&](size_t n) {
    raw.assign(n + 64, 0);
    const size_t off = (64 - reinterpret_cast<uintptr_t>(raw.data()) % 64) % 64;
    buf = raw.data() + off;
    buf_len = n;
  };
  std::string line;
  while (std::getline(std::cin, line)) {
    std::istringstream in(line);
    std::string cmd;
    if (!(in >> cmd)) continue;
    if (cmd == "region") {
      size_t n;
      in >> n;
      set_region(n);
      std::cout << "ok\n";
    } else if (cmd == "load") {
      std::string path;
      in >> path;
      std::ifstream f(path, std::ios::binary);
      std::vector<char> bytes((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
      set_region(bytes.size());
      std::memcpy(buf, bytes.data(), bytes.size());
      std::cout << "ok\n";
    } else if (cmd == "save") {
      std::string path;
      in >> path;
      std::ofstream f(path, std::ios::binary);
      f.write(reinterpret_cast<const char*>(buf), std::streamsize(buf_len));
      std::cout << "ok\n";
    } else if (cmd == "poke") {
      size_t off;
      std::string h;
      in >> off >> h;
      const std::string b = unhex(h);
      std::memcpy(buf + off, b.data(), b.size());
      std::cout << "ok\n";
    } else if (cmd == "dump") {
      std::cout << "bytes " << hex(std::string(reinterpret_cast<const char*>(buf), buf_len)) << "\n";
    } else if (cmd == "format" || cmd == "attach") {
      int nb;
      std::string uid, off_s;
      size_t len = 0;
      in >> nb >> uid;
      absl::Span<uint8_t> span(buf, buf_len);
      if (in >> off_s) {
        if (off_s == "null") {
          span = absl::Span<uint8_t>();
        } else {
          in >> len;
          span = span.subspan(std::stoul(off_s), len);
        }
      }
      auto r = cmd == "format" ? KVCacheMetadata::Format(span, nb, unhex(uid))
                               : KVCacheMetadata::Attach(span, nb, unhex(uid));
      if (r.ok()) meta = *r;
      report(r.status());
    } else if (cmd == "set") {
      int id;
      std::string h;
      uint64_t seq;
      in >> id >> h >> seq;
      report(meta->Set(id, unhex(h), seq));
    } else if (cmd == "clear") {
      int id;
      in >> id;
      report(meta->Clear(id));
    } else if (cmd == "entries") {
      for (const auto& e : meta->ValidEntries())
        std::cout << "entry " << e.block_id << " " << hex(e.hash) << " " << e.seq << "\n";
      std::cout << "end\n";
    } else if (cmd == "shm") {
      std::string key, uid;
      int nb;
      in >> key >> nb >> uid;
      auto r = KVCacheMetadataShmRegion::AttachOrFormat(key, nb, unhex(uid));
      if (!r.ok()) {
        report(r.status());
        continue;
      }
      shm = std::move(*r);
      meta = shm->metadata();
      std::cout << "ok warm=" << (shm->warm() ? 1 : 0) << "\n";
    } else if (cmd == "shm_reformat") {
      absl::Status s = shm->Reformat();
      if (s.ok()) meta = shm->metadata();
      report(s);
    } else if (cmd == "shm_close") {
      meta.reset();
      shm.reset();
      std::cout << "ok\n";
    } else {
      std::cout << "err -1 unknown command " << cmd << "\n";
    }
    std::cout.flush();
  }
  return 0;
}
