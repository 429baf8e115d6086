// Data-only reader for PyTorch ZIP checkpoints (torch.save of a whole module), and the
// MH1 converter that turns one into PWMH1001 archive bytes.
//
// The reference ships the same two pieces as a private package (checkpoint/include/
// checkpoint/checkpoint.hpp, checkpoint/src/checkpoint.cpp) and a converter
// (mace/src/weights.cpp:305-393).  This build keeps their observable contract:
//
// * ZIP: stored and deflated records, ZIP64 end records and extra fields, CRC-32 checks, one
//   PyTorch root directory; encrypted or split archives and other compressions are errors.
// * Pickle: a bounded interpreter for the opcodes protocol 2 emits.  Class and reducer names
//   become inert records: nothing is imported, constructed or called.  Tensors are rebuilt
//   as (storage, offset, shape, stride) views over the archive's storage records.
// * Errors throw std::runtime_error with "checkpoint: " (reader) or
//   "unsupported MH1 checkpoint: " (converter) prefixes, as the reference does.
#pragma once
#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace mace {
namespace ckpt {

// One strided view of a storage record.  dtype is the storage class name
// ("FloatStorage", "DoubleStorage", "LongStorage", "IntStorage", "ByteStorage",
// "BoolStorage").
struct Tensor {
  std::string dtype;
  std::shared_ptr<const std::vector<char>> storage;
  int64_t offset = 0;
  std::vector<int64_t> shape, stride;
  // Elements in row-major order of `shape`, widened to double; throws on bad metadata, a
  // view outside its storage or a nonfinite value.
  std::vector<double> values() const;
};

struct Node;
using NodeRef = std::shared_ptr<Node>;

// A decoded pickle value.  Python ints, floats and bools are numbers; str and bytes are
// text; tuples, lists and sets are items; dicts are fields.  A Global is a "module name"
// label; an Instance is the record a reducer would have built: its label, its arguments
// (items) and its state (fields).
struct Node {
  enum Kind { None, Number, Text, Items, Fields, Global, Instance, TensorView } kind = None;
  double number = 0;
  std::string text;
  std::vector<NodeRef> items;
  std::map<std::string, NodeRef> fields;
  Tensor tensor;

  const NodeRef &item(size_t i) const;
  const NodeRef &field(const std::string &key) const;
  int64_t integer() const; // exact integers only

  Node() = default;
  Node(const Node &) = default;
  Node &operator=(const Node &) = default;
  // Releases nested values iteratively: a pickle can nest containers far deeper than the
  // call stack would allow a recursive release to go.
  ~Node();
};

class Zip {
public:
  explicit Zip(const std::string &path);
  explicit Zip(std::vector<char> bytes);
  // Decompressed, CRC-checked contents of `name` (relative to the root directory).
  std::vector<char> read(const std::string &name) const;
  std::vector<std::string> names() const;
  bool has(const std::string &name) const;

private:
  struct Entry {
    uint16_t method = 0;
    uint32_t crc = 0;
    uint64_t packed = 0, size = 0, header = 0;
  };
  void scan();
  uint64_t le(uint64_t at, unsigned bytes) const;
  std::vector<char> bytes_;
  std::map<std::string, Entry> entries_;
};

// Decode one pickle; persistent storage references resolve to `zip`'s data/<key> records.
NodeRef unpickle(const std::vector<char> &pickle, const Zip &zip);
// The checkpoint's root object (data.pkl), after the byteorder check.
NodeRef load(const Zip &zip);

// Module attribute lookup: the object's own state first, then its _parameters, _buffers
// and _modules dictionaries.
const NodeRef &member(const NodeRef &object, const std::string &name);
// Dotted walk of member(): "interactions.0.linear_up".
NodeRef walk(const NodeRef &object, const std::string &dotted);
// Every tensor reachable through _parameters/_buffers/_modules, keyed by dotted name.
std::map<std::string, Tensor> tensors(const NodeRef &object);

bool is_zip(const std::string &path);

} // namespace ckpt

// The PWMH1001 archive bytes for `path`: the file itself when it is an archive (where a
// non-empty head is an error), else the conversion of a ScaleShiftMACE MH1 checkpoint for
// `head` ("matpes_r2scan" when empty).
std::string weight_data(const std::string &path, const std::string &head);
// The conversion alone, from the bytes of a ZIP checkpoint already in memory.
std::string convert_checkpoint(std::vector<char> zip_bytes, const std::string &head);

} // namespace mace
