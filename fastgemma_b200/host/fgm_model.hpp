// .fgm model files on the CUDA backend: the reference's fgm-core Model
// (src/model.rs:1-222) restated in C++ over the C ABI.  A .fgm file
// (written by convert/fgm.py) is
//
//   [0, 8)    magic "FASTGEM1"
//   [8, 12)   u32 little-endian header length
//   [12, ..)  JSON header {"arch", "config", "meta", "tensors"}; every tensor
//             entry holds {dtype, shape, offset, nbytes, meta}
//   ...       tensor blobs, 64-byte aligned, already in the kernels' layouts
//
// Model::open maps the file and parses the header; nothing is copied or
// repacked.  Quantised linears resolve like model.rs:169-208: "<name>" is a
// q4g or q8c blob of shape [N, K] whose meta carries "group" (int4 scale
// group, default 64) and "hadamard" (block size folded into the weight, 0 =
// none); "<name>.scale" holds f16 [K/group][N] or f32 [N] scales;
// "<name>.i8" is the optional int8 twin.  Where the Rust code panics (bad
// magic, a missing tensor, a non-linear dtype) this layer throws
// fgm_kernels::Error.
//
// On this backend loading also means residency: register_linears() copies
// every quantised weight and its scales into the device registry
// (fgm_cuda_register), so GEMMs given these host addresses read the device
// copies, with no host-to-device traffic per call.
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "fgm_host.hpp"

namespace fgm_core {

// A JSON value: the header's subset of JSON (objects, arrays, strings,
// numbers, booleans, null).
struct Json {
  enum Kind { Null, Bool, Number, String, Array, Object };
  Kind kind = Null;
  bool b = false;
  double num = 0.0;
  std::string str;
  std::vector<Json> arr;
  std::map<std::string, Json> obj;

  // Object member `key`, or nullptr (also when this is not an object).
  const Json *find(const std::string &key) const;
  // Parse `len` bytes of UTF-8 JSON; throws fgm_kernels::Error on bad input.
  static Json parse(const char *text, size_t len);
};

// model.rs:14-22
struct TensorEntry {
  std::string dtype;
  std::vector<size_t> shape;
  size_t offset = 0, nbytes = 0;
  Json meta;
};

class Model {
 public:
  // model.rs:117-127: map `path`, check the magic, parse the header.  Also
  // checks that every tensor lies inside the file.
  static std::unique_ptr<Model> open(const std::string &path);
  ~Model();
  Model(const Model &) = delete;
  Model &operator=(const Model &) = delete;

  bool has(const std::string &name) const;                // model.rs:129-131
  const TensorEntry &entry(const std::string &name) const;  // throws: missing tensor
  const std::vector<size_t> &shape(const std::string &name) const;

  // Typed views of a tensor's bytes (model.rs:138-163).
  fgm_kernels::Slice<const uint8_t> u8s(const std::string &name) const;
  fgm_kernels::Slice<const int8_t> i8s(const std::string &name) const;
  fgm_kernels::Slice<const fgm_kernels::f16> f16s(const std::string &name) const;
  fgm_kernels::Slice<const float> f32s(const std::string &name) const;

  QLinear linear(const std::string &name) const;  // model.rs:169-194
  DualW dual(const std::string &name) const;      // model.rs:196-208
  size_t total_bytes() const;                     // model.rs:219-221

  const Json &config() const { return config_; }
  const Json &meta() const { return meta_; }
  const std::map<std::string, TensorEntry> &tensors() const { return tensors_; }
  size_t file_bytes() const { return size_; }

  // Make every q4g / q8c tensor and its "<name>.scale" resident on the
  // device (fgm_cuda_register); returns the bytes registered.  Call
  // unregister_linears() before the Model is destroyed if the process keeps
  // using the device.
  size_t register_linears() const;
  void unregister_linears() const;

 private:
  Model() = default;
  const uint8_t *raw(const std::string &name, size_t *nbytes) const;

  const uint8_t *base_ = nullptr;
  size_t size_ = 0;
  Json config_, meta_;
  std::map<std::string, TensorEntry> tensors_;
};

}  // namespace fgm_core
