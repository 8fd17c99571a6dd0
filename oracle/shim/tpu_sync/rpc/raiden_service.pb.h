// Stand-in for the generated message classes that the reference's
// pool_layout.cc and pool reshard planner sources name (RegionSpecProto,
// PoolSpecProto, RaidenIdProto, VariableMetadataProto,
// RegisterWorkUnitRequest), used ONLY to compile those sources as test
// oracles (oracle/build_ref.py).  Plain accessors with the field names of the
// reference's proto; nothing here is generated code.
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

class RaidenIdProto {
 public:
  void set_job_name(const std::string& v) { job_name_ = v; }
  void set_job_replica_id(const std::string& v) { job_replica_id_ = v; }
  void set_data_name(const std::string& v) { data_name_ = v; }
  void set_data_replica_idx(int32_t v) { data_replica_idx_ = v; }
  const std::string& job_name() const { return job_name_; }
  const std::string& job_replica_id() const { return job_replica_id_; }
  const std::string& data_name() const { return data_name_; }
  int32_t data_replica_idx() const { return data_replica_idx_; }

 private:
  std::string job_name_, job_replica_id_, data_name_;
  int32_t data_replica_idx_ = 0;
};

// Variable metadata rides along in registrations; the planner never reads it.
class VariableMetadataProto {};

class RegisterWorkUnitRequest {
 public:
  const RaidenIdProto& unit() const { return unit_; }
  RaidenIdProto* mutable_unit() { return &unit_; }
  void add_shards(const std::string& v) { shards_.push_back(v); }
  const std::string& shards(int i) const { return shards_[size_t(i)]; }
  int shards_size() const { return int(shards_.size()); }
  void set_control_plane_rpc_address(const std::string& v) { ctl_ = v; }
  const std::string& control_plane_rpc_address() const { return ctl_; }
  void set_itemsize(int32_t v) { itemsize_ = v; }
  int32_t itemsize() const { return itemsize_; }
  void set_layout_fingerprint(const std::string& v) { fp_ = v; }
  const std::string& layout_fingerprint() const { return fp_; }
  void set_page_tokens(int64_t v) { page_tokens_ = v; }
  int64_t page_tokens() const { return page_tokens_; }
  void set_transfer_parallelism(int32_t v) { par_ = v; }
  int32_t transfer_parallelism() const { return par_; }
  void set_transfer_rank(int32_t v) { rank_ = v; }
  int32_t transfer_rank() const { return rank_; }
  void add_mesh_shape(int64_t v) { mesh_shape_.push_back(v); }
  void add_layout(int32_t v) { layout_.push_back(v); }
  void add_global_shape(int64_t v) { global_shape_.push_back(v); }
  PoolSpecProto* add_pools() { pools_.emplace_back(); return &pools_.back(); }
  const std::vector<PoolSpecProto>& pools() const { return pools_; }
  const PoolSpecProto& pools(int i) const { return pools_[size_t(i)]; }
  int pools_size() const { return int(pools_.size()); }
  VariableMetadataProto* add_variables() { variables_.emplace_back(); return &variables_.back(); }

 private:
  RaidenIdProto unit_;
  std::vector<std::string> shards_;
  std::string ctl_, fp_;
  int32_t itemsize_ = 0, par_ = 0, rank_ = 0;
  int64_t page_tokens_ = 0;
  std::vector<int64_t> mesh_shape_, global_shape_;
  std::vector<int32_t> layout_;
  std::vector<PoolSpecProto> pools_;
  std::vector<VariableMetadataProto> variables_;
};

}  // namespace rpc
}  // namespace tpu_sync
