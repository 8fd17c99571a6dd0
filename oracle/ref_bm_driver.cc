// Test driver around the REFERENCE LogicalBlockManager
// (tpu_sync/kv_cache/logical_block_manager.cc), compiled from the reference
// checkout by oracle/build_ref.py into oracle/_ref/bm_ref.  TEST
// INFRASTRUCTURE ONLY.  Reads one operation per line on stdin and prints one
// result line:
//
//   new N                      -> "ok"            (a fresh manager of N blocks)
//   alloc K L                  -> "<code> <ids>"  (Allocate(K, lock = L))
//   target|unlock|dealloc ids  -> "<code>"        (AllocateTarget / Unlock / Deallocate)
//   access ID                  -> "<code>"        (AccessBlock)
//   stats                      -> "<free> <allocated> <locked>"
//
// <code> is absl::StatusCode's number (0 = OK); <ids> is "-" on error.
#include <iostream>
#include <memory>
#include <sstream>
#include <string>
#include <vector>

#include "tpu_sync/kv_cache/logical_block_manager.h"

int main() {
  std::unique_ptr<tpu_raiden::kv_cache::LogicalBlockManager> bm;
  std::string line;
  while (std::getline(std::cin, line)) {
    std::istringstream in(line);
    std::string op;
    in >> op;
    if (op == "new") {
      int n = 0;
      in >> n;
      bm = std::make_unique<tpu_raiden::kv_cache::LogicalBlockManager>(n);
      std::cout << "ok\n";
    } else if (op == "alloc") {
      int k = 0, lock = 0;
      in >> k >> lock;
      auto r = bm->Allocate(k, lock != 0);
      std::cout << static_cast<int>(r.status().code());
      if (r.ok()) {
        for (int id : *r) std::cout << " " << id;
      } else {
        std::cout << " -";
      }
      std::cout << "\n";
    } else if (op == "target" || op == "unlock" || op == "dealloc") {
      std::vector<int> ids;
      int id;
      while (in >> id) ids.push_back(id);
      absl::Span<const int> span(ids.data(), ids.size());
      absl::Status s = op == "target"   ? bm->AllocateTarget(span)
                       : op == "unlock" ? bm->Unlock(span)
                                        : bm->Deallocate(span);
      std::cout << static_cast<int>(s.code()) << "\n";
    } else if (op == "access") {
      int id = 0;
      in >> id;
      std::cout << static_cast<int>(bm->AccessBlock(id).code()) << "\n";
    } else if (op == "stats") {
      std::cout << bm->num_free_blocks() << " " << bm->num_allocated_blocks() << " "
                << bm->num_locked_blocks() << "\n";
    } else if (!op.empty()) {
      std::cout << "?\n";
    }
  }
  return 0;
}
