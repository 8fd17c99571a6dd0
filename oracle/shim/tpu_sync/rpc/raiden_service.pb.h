// Stand-in for the two generated message classes pool_layout.h names
// (RegionSpecProto / PoolSpecProto), used ONLY to compile the reference's
// pool_layout.cc as a test oracle (oracle/build_ref.py).  Plain accessors with
// the field names of the reference's proto; nothing here is generated code.
#pragma once
#include <cstdint>
#include <string>
#include <vector>

namespace tpu_sync {
namespace rpc {

class RegionSpecProto {
 public:
  void set_name(const std::string& v) { name_ = v; }
  void set_offset_bytes(int64_t v) { offset_ = v; }
  void set_stride_bytes(int64_t v) { stride_ = v; }
  void set_unit_bytes(int64_t v) { unit_ = v; }
  void set_num_units(int64_t v) { num_ = v; }
  void set_units_per_stride(int64_t v) { ups_ = v; }
  const std::string& name() const { return name_; }
  int64_t offset_bytes() const { return offset_; }
  int64_t stride_bytes() const { return stride_; }
  int64_t unit_bytes() const { return unit_; }
  int64_t num_units() const { return num_; }
  int64_t units_per_stride() const { return ups_; }

 private:
  std::string name_;
  int64_t offset_ = 0, stride_ = 0, unit_ = 0, num_ = 0, ups_ = 0;
};

class PoolSpecProto {
 public:
  void set_tag(const std::string& v) { tag_ = v; }
  void set_storage_index(int64_t v) { storage_ = v; }
  void set_base_offset_bytes(int64_t v) { base_ = v; }
  void set_block_stride_bytes(int64_t v) { stride_ = v; }
  void set_num_blocks(int64_t v) { nb_ = v; }
  void set_dtype_tag(const std::string& v) { dtype_ = v; }
  RegionSpecProto* add_regions() { regions_.emplace_back(); return &regions_.back(); }
  const std::string& tag() const { return tag_; }
  int64_t storage_index() const { return storage_; }
  int64_t base_offset_bytes() const { return base_; }
  int64_t block_stride_bytes() const { return stride_; }
  int64_t num_blocks() const { return nb_; }
  const std::string& dtype_tag() const { return dtype_; }
  const std::vector<RegionSpecProto>& regions() const { return regions_; }
  int regions_size() const { return int(regions_.size()); }

 private:
  std::string tag_, dtype_;
  int64_t storage_ = 0, base_ = 0, stride_ = 0, nb_ = 0;
  std::vector<RegionSpecProto> regions_;
};

}  // namespace rpc
}  // namespace tpu_sync
