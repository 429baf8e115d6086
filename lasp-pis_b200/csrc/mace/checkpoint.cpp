// PyTorch ZIP checkpoint reader: ZIP directory, deflate via zlib, and a data-only pickle
// interpreter.  Behaviour and limits follow the reference reader
// (checkpoint/src/checkpoint.cpp:61-253 for the ZIP layer, 255-328 for tensor views,
// 330-657 for the pickle opcodes, 658-715 for module lookup), so that the same files are
// accepted and the same malformed ones rejected.
#include "checkpoint.hpp"
#include <cmath>
#include <cstring>
#include <fstream>
#include <functional>
#include <limits>
#include <set>
#include <stdexcept>
#include <zlib.h>

namespace mace {
namespace ckpt {
namespace {

[[noreturn]] void fail(const std::string &what) { throw std::runtime_error("checkpoint: " + what); }

constexpr uint32_t kLocalHeader = 0x04034b50, kCentralHeader = 0x02014b50, kEnd = 0x06054b50,
                   kEnd64 = 0x06064b50, kLocator64 = 0x07064b50;
constexpr uint64_t kArchiveLimit = uint64_t(1) << 31, kRecordLimit = uint64_t(1) << 30;
constexpr size_t kPickleLimit = size_t(32) << 20, kStorageLimit = size_t(1) << 31;
constexpr size_t kOpLimit = 10000000, kStackLimit = 1000000, kMarkLimit = 10000, kMemoLimit = 1000000;
constexpr uint64_t kMaxElements = uint64_t(1) << 27;

NodeRef make(Node::Kind kind) {
  auto n = std::make_shared<Node>();
  n->kind = kind;
  return n;
}
NodeRef number(double x) {
  auto n = make(Node::Number);
  n->number = x;
  return n;
}

} // namespace

// ----------------------------------------------------------------------------------- Node

const NodeRef &Node::item(size_t i) const {
  if (i >= items.size())
    fail("sequence index out of range on " + text);
  return items[i];
}

const NodeRef &Node::field(const std::string &key) const {
  auto it = fields.find(key);
  if (it == fields.end())
    fail("missing attribute " + key + " on " + text);
  return it->second;
}

Node::~Node() {
  std::vector<NodeRef> pending;
  auto detach = [&pending](Node &n) {
    for (auto &x : n.items)
      pending.push_back(std::move(x));
    n.items.clear();
    for (auto &kv : n.fields)
      pending.push_back(std::move(kv.second));
    n.fields.clear();
  };
  detach(*this);
  while (!pending.empty()) {
    NodeRef x = std::move(pending.back());
    pending.pop_back();
    // Only the last owner empties a node; its release below then has nothing nested left.
    if (x && x.use_count() == 1)
      detach(*x);
  }
}

int64_t Node::integer() const {
  // Exactly representable integers only (|x| < 2^53).
  if (kind != Number || !std::isfinite(number) || std::trunc(number) != number ||
      std::fabs(number) > 9007199254740991.0)
    fail("invalid integer");
  return int64_t(number);
}

// ------------------------------------------------------------------------------------ ZIP

Zip::Zip(const std::string &path) {
  std::ifstream in(path, std::ios::binary | std::ios::ate);
  if (!in)
    fail("cannot open " + path);
  auto size = in.tellg();
  if (size < 0 || uint64_t(size) > kArchiveLimit)
    fail("archive exceeds 2 GiB limit");
  bytes_.resize(size_t(size));
  in.seekg(0);
  if (!in.read(bytes_.data(), std::streamsize(bytes_.size())))
    fail("cannot read " + path);
  scan();
}

Zip::Zip(std::vector<char> bytes) : bytes_(std::move(bytes)) { scan(); }

uint64_t Zip::le(uint64_t at, unsigned width) const {
  if (at > bytes_.size() || width > bytes_.size() - at)
    fail("truncated ZIP metadata");
  uint64_t v = 0;
  for (unsigned k = width; k-- > 0;)
    v = (v << 8) | uint8_t(bytes_[size_t(at + k)]);
  return v;
}

void Zip::scan() {
  const uint64_t n = bytes_.size();
  if (n < 22 || n > kArchiveLimit)
    fail("invalid ZIP size");
  // The end record is the last 22 bytes plus a comment of at most 64 KiB whose length it
  // states; search backwards for a signature whose comment reaches the end of the file.
  uint64_t end = n - 22;
  const uint64_t lowest = end > 65535 ? end - 65535 : 0;
  for (;; --end) {
    if (le(end, 4) == kEnd && end + 22 + le(end + 20, 2) == n)
      break;
    if (end == lowest)
      fail("missing ZIP end record");
  }
  if (le(end + 4, 2) != 0 || le(end + 6, 2) != 0)
    fail("split ZIP archives are unsupported");
  uint64_t count = le(end + 10, 2), dir_size = le(end + 12, 4), dir_at = le(end + 16, 4);
  if (count == 0xffff || dir_size == 0xffffffff || dir_at == 0xffffffff) {
    // ZIP64: a 20-byte locator right before the end record points at the 64-bit end record.
    if (end < 20 || le(end - 20, 4) != kLocator64 || le(end - 16, 4) != 0 || le(end - 4, 4) != 1)
      fail("invalid ZIP64 locator");
    const uint64_t e64 = le(end - 12, 8);
    if (le(e64, 4) != kEnd64 || le(e64 + 4, 8) < 44 || le(e64 + 16, 4) != 0 || le(e64 + 20, 4) != 0)
      fail("invalid ZIP64 end record");
    count = le(e64 + 32, 8);
    dir_size = le(e64 + 40, 8);
    dir_at = le(e64 + 48, 8);
    if (le(e64 + 24, 8) != count)
      fail("inconsistent ZIP64 entry counts");
  } else if (le(end + 8, 2) != count) {
    fail("inconsistent ZIP entry counts");
  }
  if (count > 100000 || dir_at > end || dir_size > end - dir_at)
    fail("invalid ZIP central directory");

  const uint64_t dir_end = dir_at + dir_size;
  uint64_t at = dir_at;
  std::string root;
  for (uint64_t k = 0; k < count; ++k) {
    if (at > dir_end || dir_end - at < 46 || le(at, 4) != kCentralHeader)
      fail("invalid ZIP entry");
    if (le(at + 8, 2) & 1)
      fail("encrypted ZIP is unsupported");
    Entry e;
    e.method = uint16_t(le(at + 10, 2));
    e.crc = uint32_t(le(at + 16, 4));
    e.packed = le(at + 20, 4);
    e.size = le(at + 24, 4);
    e.header = le(at + 42, 4);
    const uint64_t name_len = le(at + 28, 2), extra_len = le(at + 30, 2), comment_len = le(at + 32, 2);
    if (name_len + extra_len + comment_len > dir_end - at - 46)
      fail("truncated ZIP entry");
    std::string name(bytes_.data() + at + 46, size_t(name_len));

    // Saturated 32-bit fields are replaced, in the order size, packed size, header offset,
    // from the ZIP64 extra field (tag 1).
    uint64_t *wanted[3] = {e.size == 0xffffffff ? &e.size : nullptr,
                           e.packed == 0xffffffff ? &e.packed : nullptr,
                           e.header == 0xffffffff ? &e.header : nullptr};
    for (uint64_t x = at + 46 + name_len, xend = x + extra_len; x < xend;) {
      if (xend - x < 4)
        fail("invalid ZIP extra field");
      const uint64_t tag = le(x, 2), len = le(x + 2, 2);
      x += 4;
      if (len > xend - x)
        fail("truncated ZIP extra field");
      if (tag == 1) {
        uint64_t q = x;
        for (auto &slot : wanted)
          if (slot) {
            if (x + len - q < 8)
              fail("truncated ZIP64 extra field");
            *slot = le(q, 8);
            q += 8;
            slot = nullptr;
          }
      }
      x += len;
    }
    if (wanted[0] || wanted[1] || wanted[2] || le(at + 34, 2) != 0)
      fail("unsupported ZIP64 entry");
    if (e.method != 0 && e.method != 8)
      fail("unsupported ZIP compression");
    if (e.size > kRecordLimit || e.header > dir_at || dir_at - e.header < 30)
      fail("invalid ZIP record bounds");

    // torch.save puts every record under one root directory (named after the file).
    const auto slash = name.find('/');
    if (slash == std::string::npos || slash == 0)
      fail("expected PyTorch ZIP root directory");
    if (root.empty())
      root = name.substr(0, slash + 1);
    if (name.compare(0, root.size(), root) != 0)
      fail("inconsistent ZIP root");
    if (!entries_.emplace(name.substr(root.size()), e).second)
      fail("duplicate ZIP record: " + name.substr(root.size()));
    at += 46 + name_len + extra_len + comment_len;
  }
  if (at != dir_end)
    fail("trailing ZIP directory data");
}

bool Zip::has(const std::string &name) const { return entries_.count(name) != 0; }

std::vector<std::string> Zip::names() const {
  std::vector<std::string> out;
  out.reserve(entries_.size());
  for (const auto &kv : entries_)
    out.push_back(kv.first);
  return out;
}

std::vector<char> Zip::read(const std::string &name) const {
  auto it = entries_.find(name);
  if (it == entries_.end())
    fail("missing ZIP record: " + name);
  const Entry &e = it->second;
  if (le(e.header, 4) != kLocalHeader || (le(e.header + 6, 2) & 1) || le(e.header + 8, 2) != e.method)
    fail("invalid local ZIP header");
  const uint64_t begin = e.header + 30 + le(e.header + 26, 2) + le(e.header + 28, 2);
  if (begin > bytes_.size() || e.packed > bytes_.size() - begin)
    fail("truncated ZIP record");
  std::vector<char> out(size_t(e.size));
  if (e.method == 0) {
    if (e.packed != e.size)
      fail("stored ZIP size mismatch");
    if (e.size)
      std::memcpy(out.data(), bytes_.data() + begin, size_t(e.size));
  } else {
    // Raw deflate (no zlib header); the stream must end exactly at both stated sizes.
    unsigned char sink = 0;
    z_stream z{};
    z.next_in = reinterpret_cast<Bytef *>(const_cast<char *>(bytes_.data() + begin));
    z.avail_in = uInt(e.packed);
    z.next_out = out.empty() ? &sink : reinterpret_cast<Bytef *>(out.data());
    z.avail_out = out.empty() ? 1u : uInt(out.size());
    if (inflateInit2(&z, -MAX_WBITS) != Z_OK)
      fail("cannot initialize ZIP decompression");
    const int status = inflate(&z, Z_FINISH);
    const uint64_t produced = z.total_out, consumed = z.total_in;
    inflateEnd(&z);
    if (status != Z_STREAM_END || produced != e.size || consumed != e.packed)
      fail("invalid compressed ZIP data");
  }
  const uLong crc = crc32(0L, reinterpret_cast<const Bytef *>(out.data()), uInt(out.size()));
  if (crc != e.crc)
    fail("ZIP checksum mismatch: " + name);
  return out;
}

bool is_zip(const std::string &path) {
  std::ifstream in(path, std::ios::binary);
  if (!in)
    fail("cannot open " + path);
  char head[4] = {};
  in.read(head, 4);
  return std::memcmp(head, "PK\x03\x04", 4) == 0;
}

// ---------------------------------------------------------------------------- tensor view

namespace {
template <class T> double widen(const char *p) {
  T x;
  std::memcpy(&x, p, sizeof(T));
  return double(x);
}
} // namespace

std::vector<double> Tensor::values() const {
  if (!storage || shape.size() != stride.size() || shape.size() > 8 || offset < 0)
    fail("invalid tensor metadata");
  size_t width;
  double (*read)(const char *);
  if (dtype == "FloatStorage")
    width = 4, read = widen<float>;
  else if (dtype == "DoubleStorage")
    width = 8, read = widen<double>;
  else if (dtype == "LongStorage")
    width = 8, read = widen<int64_t>;
  else if (dtype == "IntStorage")
    width = 4, read = widen<int32_t>;
  else if (dtype == "BoolStorage" || dtype == "ByteStorage")
    width = 1, read = widen<uint8_t>;
  else
    fail("unsupported tensor dtype " + dtype);
  uint64_t total = 1;
  for (size_t d = 0; d < shape.size(); ++d) {
    if (shape[d] < 0 || stride[d] < 0 || uint64_t(shape[d]) > kMaxElements ||
        (shape[d] && total > kMaxElements / uint64_t(shape[d])))
      fail("invalid tensor shape or stride");
    total *= uint64_t(shape[d]);
  }
  std::vector<double> out(static_cast<size_t>(total));
  if (total == 0)
    return out;
  // Strides are non-negative, so the last element of the view is the farthest one: bound it
  // once instead of every element.
  uint64_t last = uint64_t(offset);
  for (size_t d = 0; d < shape.size(); ++d) {
    const uint64_t c = uint64_t(shape[d] - 1);
    if (c && uint64_t(stride[d]) > (std::numeric_limits<uint64_t>::max() - last) / c)
      fail("tensor offset overflow");
    last += c * uint64_t(stride[d]);
  }
  if (last >= storage->size() / width)
    fail("tensor exceeds storage");
  const char *base = storage->data() + size_t(offset) * width;
  bool dense = true;
  for (size_t d = shape.size(), step = 1; d-- > 0; step *= size_t(shape[d]))
    dense = dense && (shape[d] == 1 || size_t(stride[d]) == step);
  if (dense) {
    for (size_t i = 0; i < out.size(); ++i)
      out[i] = read(base + i * width);
  } else {
    // Odometer over the shape, tracking the element offset incrementally.
    std::vector<int64_t> idx(shape.size(), 0);
    uint64_t at = 0;
    for (size_t i = 0; i < out.size(); ++i) {
      out[i] = read(base + at * width);
      for (size_t d = shape.size(); d-- > 0;) {
        at += uint64_t(stride[d]);
        if (++idx[d] < shape[d])
          break;
        at -= uint64_t(stride[d]) * uint64_t(shape[d]);
        idx[d] = 0;
      }
    }
  }
  for (double v : out)
    if (!std::isfinite(v))
      fail("nonfinite tensor value");
  return out;
}

// --------------------------------------------------------------------------------- pickle

namespace {

class Machine {
public:
  Machine(const std::vector<char> &code, const Zip &zip) : code_(code), zip_(zip) {}

  NodeRef run() {
    if (code_.size() > kPickleLimit)
      fail("pickle record too large");
    size_t ops = 0;
    while (pos_ < code_.size()) {
      if (++ops > kOpLimit || stack_.size() > kStackLimit || marks_.size() > kMarkLimit)
        fail("pickle resource limit");
      const unsigned op = u8();
      if (op == '.') {
        if (stack_.size() != 1 || !marks_.empty() || pos_ != code_.size())
          fail("invalid pickle end");
        return stack_[0];
      }
      step(op);
    }
    fail("pickle has no STOP");
  }

private:
  const std::vector<char> &code_;
  const Zip &zip_;
  size_t pos_ = 0;
  std::vector<NodeRef> stack_, memo_;
  std::vector<size_t> marks_;
  std::map<std::string, std::shared_ptr<const std::vector<char>>> storages_;
  size_t storage_bytes_ = 0;

  unsigned u8() {
    if (pos_ >= code_.size())
      fail("truncated pickle");
    return uint8_t(code_[pos_++]);
  }
  uint64_t uint_le(int n) {
    uint64_t v = 0;
    for (int k = 0; k < n; ++k)
      v |= uint64_t(u8()) << (8 * k);
    return v;
  }
  std::string take(uint64_t n) {
    if (n > code_.size() - pos_)
      fail("truncated string");
    std::string s(code_.data() + pos_, size_t(n));
    pos_ += size_t(n);
    return s;
  }
  std::string text_line() {
    const size_t start = pos_;
    while (pos_ < code_.size() && code_[pos_] != '\n')
      ++pos_;
    if (pos_ == code_.size())
      fail("truncated global");
    std::string s(code_.data() + start, pos_ - start);
    ++pos_;
    return s;
  }
  void push(NodeRef n) { stack_.push_back(std::move(n)); }
  NodeRef pop() {
    if (stack_.empty())
      fail("pickle stack underflow");
    NodeRef n = std::move(stack_.back());
    stack_.pop_back();
    return n;
  }
  size_t pop_mark() {
    if (marks_.empty())
      fail("missing pickle mark");
    const size_t m = marks_.back();
    marks_.pop_back();
    if (m > stack_.size())
      fail("invalid mark");
    return m;
  }
  // Replace the top n stack entries by one Items node holding them.
  void collect(size_t n) {
    if (n > stack_.size())
      fail("tuple underflow");
    auto t = make(Node::Items);
    t->items.assign(stack_.end() - std::ptrdiff_t(n), stack_.end());
    stack_.resize(stack_.size() - n);
    push(std::move(t));
  }
  static std::string key_of(const NodeRef &k) {
    if (k->kind == Node::Text)
      return k->text;
    if (k->kind == Node::Number)
      return std::to_string(k->integer());
    fail("unsupported dictionary key");
  }
  // Move stack[from:] into `dict` as key, value pairs.
  void fill(const NodeRef &dict, size_t from) {
    if ((stack_.size() - from) % 2)
      fail("odd dictionary payload");
    for (size_t k = from; k < stack_.size(); k += 2)
      dict->fields[key_of(stack_[k])] = stack_[k + 1];
    stack_.resize(from);
  }
  void memo_store(uint64_t index) {
    if (index > kMemoLimit || stack_.empty())
      fail("invalid memo");
    if (memo_.size() <= index)
      memo_.resize(size_t(index) + 1);
    memo_[size_t(index)] = stack_.back();
  }
  void memo_fetch(uint64_t index) {
    if (index >= memo_.size() || !memo_[size_t(index)])
      fail("invalid memo reference");
    push(memo_[size_t(index)]);
  }

  // BINPERSID: ('storage', <storage class>, key, location, numel) -> a flat view.
  NodeRef storage(const NodeRef &pid) {
    if (pid->items.size() < 5 || pid->item(0)->text != "storage")
      fail("unsupported persistent reference");
    std::string dtype = pid->item(1)->text;
    dtype = dtype.substr(dtype.find_last_of(' ') + 1);
    const std::string &key = pid->item(2)->text;
    if (key.find_first_not_of("0123456789") != std::string::npos)
      fail("invalid storage key");
    auto &slot = storages_[key];
    if (!slot) {
      auto bytes = std::make_shared<std::vector<char>>(zip_.read("data/" + key));
      storage_bytes_ += bytes->size();
      if (storage_bytes_ > kStorageLimit)
        fail("checkpoint storage limit");
      slot = std::move(bytes);
    }
    auto t = make(Node::TensorView);
    t->tensor.storage = slot;
    t->tensor.dtype = dtype;
    t->tensor.shape = {pid->item(4)->integer()};
    t->tensor.stride = {1};
    return t;
  }

  static std::vector<int64_t> int_list(const NodeRef &n) {
    std::vector<int64_t> v;
    v.reserve(n->items.size());
    for (const auto &x : n->items)
      v.push_back(x->integer());
    return v;
  }

  // REDUCE / NEWOBJ.  A few torch and stdlib reducers are interpreted as data; every other
  // callable becomes an inert Instance record.
  NodeRef reduce(const NodeRef &callable, const NodeRef &args) {
    if (callable->kind != Node::Global)
      fail("invalid constructor");
    const std::string &name = callable->text;
    if (name == "collections OrderedDict") {
      auto d = make(Node::Fields);
      if (!args->items.empty())
        for (const auto &pair : args->item(0)->items)
          d->fields[key_of(pair->item(0))] = pair->item(1);
      return d;
    }
    if (name == "torch._utils _rebuild_tensor_v2" || name == "torch._utils _rebuild_tensor") {
      auto t = make(Node::TensorView);
      t->tensor = args->item(0)->tensor;
      t->tensor.offset = args->item(1)->integer();
      t->tensor.shape = int_list(args->item(2));
      t->tensor.stride = int_list(args->item(3));
      return t;
    }
    if (name == "torch._utils _rebuild_parameter" || name == "torch._utils _rebuild_parameter_with_state" ||
        name == "torch.jit._pickle restore_type_tag")
      return args->item(0);
    if (name == "torch.jit._pickle build_intlist" || name == "torch.jit._pickle build_tensorlist" ||
        name == "__builtin__ set" || name == "builtins set")
      return args->items.empty() ? make(Node::Items) : args->item(0);
    if (name == "_codecs encode") {
      // Protocol 2 stores bytes as the UTF-8 text of their latin-1 decoding.
      if (args->item(1)->text != "latin1")
        fail("unsupported byte encoding");
      const std::string &s = args->item(0)->text;
      auto b = make(Node::Text);
      b->text.reserve(s.size());
      for (size_t i = 0; i < s.size(); ++i) {
        unsigned c = uint8_t(s[i]);
        if (c == 0xc2 || c == 0xc3) {
          if (++i >= s.size())
            fail("invalid latin1");
          c = ((c & 3u) << 6) | (uint8_t(s[i]) & 63u);
        } else if (c >= 128) {
          fail("invalid latin1");
        }
        b->text.push_back(char(c));
      }
      return b;
    }
    auto obj = make(Node::Instance);
    obj->text = name;
    obj->items = args->items;
    // e3nn irreps pickle as Cls((a, b, ...)): keep their elements as the items.
    if ((name == "e3nn.o3._irreps Irreps" || name == "e3nn.o3._irreps Irrep") && obj->items.size() == 1 &&
        obj->items[0]->kind == Node::Items) {
      auto inner = obj->items[0]->items;
      obj->items = std::move(inner);
    }
    return obj;
  }

  void step(unsigned op) {
    switch (op) {
    case 0x80: { // PROTO
      const unsigned p = u8();
      if (p < 2 || p > 5)
        fail("unsupported pickle protocol");
      break;
    }
    case 0x95: // FRAME: every read stays bounded by the record anyway
      uint_le(8);
      break;
    case '(': // MARK
      marks_.push_back(stack_.size());
      break;
    case 'N':
      push(make(Node::None));
      break;
    case 0x88: // NEWTRUE
      push(number(1));
      break;
    case 0x89: // NEWFALSE
      push(number(0));
      break;
    case 'K': // BININT1
      push(number(u8()));
      break;
    case 'M': // BININT2
      push(number(double(uint_le(2))));
      break;
    case 'J': // BININT
      push(number(int32_t(uint32_t(uint_le(4)))));
      break;
    case 0x8a: { // LONG1: little-endian two's complement of n <= 7 bytes
      const unsigned n = u8();
      if (n > 7)
        fail("integer too large");
      uint64_t v = uint_le(int(n));
      if (n && (v >> (8 * n - 1)) & 1)
        v |= ~uint64_t(0) << (8 * n);
      push(number(double(int64_t(v))));
      break;
    }
    case 'G': { // BINFLOAT: big-endian IEEE double
      uint64_t bits = 0;
      for (int k = 0; k < 8; ++k)
        bits = (bits << 8) | u8();
      double x;
      std::memcpy(&x, &bits, 8);
      push(number(x));
      break;
    }
    case 'X':    // BINUNICODE
    case 'B':    // BINBYTES
    case 0x8c:   // SHORT_BINUNICODE
    case 'C': {  // SHORT_BINBYTES
      const uint64_t n = (op == 0x8c || op == 'C') ? u8() : uint_le(4);
      auto s = make(Node::Text);
      s->text = take(n);
      push(std::move(s));
      break;
    }
    case 'c': { // GLOBAL module\nname\n
      auto g = make(Node::Global);
      std::string module = text_line();
      g->text = module + " " + text_line();
      push(std::move(g));
      break;
    }
    case 0x93: { // STACK_GLOBAL
      auto name = pop();
      auto module = pop();
      auto g = make(Node::Global);
      g->text = module->text + " " + name->text;
      push(std::move(g));
      break;
    }
    case 'q':
      memo_store(u8());
      break;
    case 'r':
      memo_store(uint_le(4));
      break;
    case 0x94: // MEMOIZE
      memo_store(memo_.size());
      break;
    case 'h':
      memo_fetch(u8());
      break;
    case 'j':
      memo_fetch(uint_le(4));
      break;
    case ')':  // EMPTY_TUPLE
    case ']':  // EMPTY_LIST
    case 0x8f: // EMPTY_SET
      push(make(Node::Items));
      break;
    case '}':
      push(make(Node::Fields));
      break;
    case 0x85:
    case 0x86:
    case 0x87: // TUPLE1..3
      collect(op - 0x84);
      break;
    case 't': // TUPLE
    case 'l': // LIST
      collect(stack_.size() - pop_mark());
      break;
    case 'd': { // DICT
      const size_t m = pop_mark();
      auto d = make(Node::Fields);
      fill(d, m);
      push(std::move(d));
      break;
    }
    case 'a': { // APPEND
      auto v = pop();
      if (stack_.empty())
        fail("append underflow");
      stack_.back()->items.push_back(std::move(v));
      break;
    }
    case 'e':    // APPENDS
    case 0x90: { // ADDITEMS
      const size_t m = pop_mark();
      if (m == 0)
        fail("append underflow");
      auto &target = stack_[m - 1]->items;
      target.insert(target.end(), stack_.begin() + std::ptrdiff_t(m), stack_.end());
      stack_.resize(m);
      break;
    }
    case 's': { // SETITEM
      auto v = pop();
      auto k = pop();
      if (stack_.empty())
        fail("setitem underflow");
      stack_.back()->fields[key_of(k)] = std::move(v);
      break;
    }
    case 'u': { // SETITEMS
      const size_t m = pop_mark();
      if (m == 0)
        fail("setitems underflow");
      fill(stack_[m - 1], m);
      break;
    }
    case 'Q': // BINPERSID
      push(storage(pop()));
      break;
    case 'R':    // REDUCE
    case 0x81: { // NEWOBJ
      auto args = pop();
      auto callable = pop();
      push(reduce(callable, args));
      break;
    }
    case 'b': { // BUILD: merge the state into the object's fields (existing keys win)
      auto state = pop();
      if (stack_.empty())
        fail("build underflow");
      auto &target = stack_.back()->fields;
      if (state->kind == Node::Fields || state->kind == Node::Instance)
        target.insert(state->fields.begin(), state->fields.end());
      else if (state->kind == Node::Items)
        for (const auto &part : state->items)
          target.insert(part->fields.begin(), part->fields.end());
      else
        fail("unsupported object state");
      break;
    }
    default:
      fail("unsupported pickle opcode " + std::to_string(op) + " at " + std::to_string(pos_ - 1));
    }
  }
};

} // namespace

NodeRef unpickle(const std::vector<char> &pickle, const Zip &zip) { return Machine(pickle, zip).run(); }

NodeRef load(const Zip &zip) {
  if (zip.has("byteorder")) {
    auto order = zip.read("byteorder");
    if (std::string(order.begin(), order.end()) != "little")
      fail("only little-endian storage is supported");
  }
  return unpickle(zip.read("data.pkl"), zip);
}

// ------------------------------------------------------------------------- module lookup

const NodeRef &member(const NodeRef &object, const std::string &name) {
  auto it = object->fields.find(name);
  if (it != object->fields.end())
    return it->second;
  for (const char *group : {"_parameters", "_buffers", "_modules"}) {
    auto g = object->fields.find(group);
    if (g == object->fields.end())
      continue;
    auto x = g->second->fields.find(name);
    if (x != g->second->fields.end())
      return x->second;
  }
  fail("missing module attribute " + name + " on " + object->text);
}

NodeRef walk(const NodeRef &object, const std::string &dotted) {
  NodeRef at = object;
  size_t start = 0;
  while (true) {
    const size_t dot = dotted.find('.', start);
    const std::string part = dotted.substr(start, dot == std::string::npos ? std::string::npos : dot - start);
    at = member(at, part);
    if (dot == std::string::npos)
      return at;
    start = dot + 1;
  }
}

std::map<std::string, Tensor> tensors(const NodeRef &object) {
  std::map<std::string, Tensor> out;
  std::set<const Node *> open;
  std::function<void(const NodeRef &, const std::string &, int)> visit = [&](const NodeRef &n,
                                                                              const std::string &prefix,
                                                                              int depth) {
    if (depth > 100 || !open.insert(n.get()).second)
      fail("cyclic module graph");
    for (const auto &[key, v] : n->fields) {
      if (key == "_parameters" || key == "_buffers") {
        for (const auto &[name, t] : v->fields)
          if (t->kind == Node::TensorView)
            out[prefix + name] = t->tensor;
      } else if (key == "_modules") {
        for (const auto &[name, m] : v->fields)
          visit(m, prefix + name + ".", depth + 1);
      }
      if (v->kind == Node::TensorView)
        out[prefix + key] = v->tensor;
      if (v->kind == Node::Instance && v->text.compare(0, 10, "__torch__.") == 0)
        visit(v, prefix + key + ".", depth + 1);
    }
    open.erase(n.get());
  };
  visit(object, "", 0);
  return out;
}

} // namespace ckpt
} // namespace mace
