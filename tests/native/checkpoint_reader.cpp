// Native test of the checkpoint reader (host only).  Pins what the reference's
// checkpoint/tests/reader.cpp pins:
//
//   checkpoint-reader ZIP       the fixture must open and its data.pkl decode to None; then
//                               inert reducers, malformed pickles and strided views are checked
//   checkpoint-reader --open F  only open F and decode its root (exit 1 if rejected)
//   checkpoint-reader --tree F  the decoded root as JSON: numbers, strings (bytes as
//                               \u00XX escapes), lists, objects; class records as
//                               {"$class", "items", "fields"}, tensors as {"$tensor", "shape"}
//   checkpoint-reader --tensors F   the root's class, then every tensor reachable through the
//                               module tree: "name [d0,d1,...] first-value" per line
//                               (what the reference's checkpoint_inspect prints)
//
// Prints one line on success; exits 1 with the error otherwise.
#include "checkpoint.hpp"

#include <cstdio>
#include <cstring>
#include <iomanip>
#include <iostream>
#include <stdexcept>
#include <string>
#include <vector>

using mace::ckpt::Node;

static void require(bool ok, const char *what) {
  if (!ok)
    throw std::runtime_error(std::string("checkpoint test failed: ") + what);
}

static void json_text(const std::string &t) {
  std::cout << '"';
  for (unsigned char c : t) {
    if (c == '"' || c == '\\')
      std::cout << '\\' << c;
    else if (c < 0x20 || c >= 0x7f) {
      char buf[8];
      std::snprintf(buf, sizeof(buf), "\\u%04x", c);
      std::cout << buf;
    } else
      std::cout << c;
  }
  std::cout << '"';
}

static void json_node(const mace::ckpt::NodeRef &n, int depth) {
  if (depth > 200)
    throw std::runtime_error("tree too deep to print");
  auto list = [&](const std::vector<mace::ckpt::NodeRef> &items) {
    std::cout << '[';
    for (size_t k = 0; k < items.size(); ++k) {
      if (k)
        std::cout << ',';
      json_node(items[k], depth + 1);
    }
    std::cout << ']';
  };
  auto dict = [&](const std::map<std::string, mace::ckpt::NodeRef> &fields) {
    std::cout << '{';
    bool first = true;
    for (const auto &[k, v] : fields) {
      if (!first)
        std::cout << ',';
      first = false;
      json_text(k);
      std::cout << ':';
      json_node(v, depth + 1);
    }
    std::cout << '}';
  };
  switch (n->kind) {
  case Node::None:
    std::cout << "null";
    break;
  case Node::Number: {
    // Always a float literal, so that -0.0 keeps its sign through a JSON parser.
    char buf[40];
    std::snprintf(buf, sizeof(buf), "%.17g", n->number);
    std::cout << buf << (std::strpbrk(buf, ".eni") ? "" : ".0");
    break;
  }
  case Node::Text:
    json_text(n->text);
    break;
  case Node::Items:
    list(n->items);
    break;
  case Node::Fields:
    dict(n->fields);
    break;
  case Node::Global:
  case Node::Instance:
    std::cout << "{\"$class\":";
    json_text(n->text);
    std::cout << ",\"items\":";
    list(n->items);
    std::cout << ",\"fields\":";
    dict(n->fields);
    std::cout << '}';
    break;
  case Node::TensorView:
    std::cout << "{\"$tensor\":";
    json_text(n->tensor.dtype);
    std::cout << ",\"shape\":[";
    for (size_t k = 0; k < n->tensor.shape.size(); ++k)
      std::cout << (k ? "," : "") << n->tensor.shape[k];
    std::cout << "]}";
    break;
  }
}

static bool rejects(const std::string &pickle, const mace::ckpt::Zip &zip) {
  try {
    mace::ckpt::unpickle(std::vector<char>(pickle.begin(), pickle.end()), zip);
  } catch (const std::exception &) {
    return true;
  }
  return false;
}

int main(int argc, char **argv) {
  try {
    if (argc == 3 && std::string(argv[1]) == "--open") {
      mace::ckpt::Zip zip{std::string(argv[2])};
      mace::ckpt::load(zip);
      return 0;
    }
    if (argc == 3 && std::string(argv[1]) == "--tree") {
      mace::ckpt::Zip zip{std::string(argv[2])};
      std::cout << std::setprecision(17);
      json_node(mace::ckpt::load(zip), 0);
      std::cout << "\n";
      return 0;
    }
    if (argc == 3 && std::string(argv[1]) == "--tensors") {
      mace::ckpt::Zip zip{std::string(argv[2])};
      auto root = mace::ckpt::load(zip);
      auto all = mace::ckpt::tensors(root);
      std::cout << std::setprecision(17) << root->text << " " << all.size() << " tensors\n";
      for (const auto &[name, t] : all) {
        auto v = t.values();
        std::cout << name << " [";
        for (auto d : t.shape)
          std::cout << d << ",";
        std::cout << "] " << (v.empty() ? 0.0 : v[0]) << "\n";
      }
      return 0;
    }
    if (argc != 2)
      throw std::runtime_error("usage: checkpoint-reader ZIP | --open FILE | --tree FILE | --tensors FILE");
    mace::ckpt::Zip zip{std::string(argv[1])};
    require(mace::ckpt::load(zip)->kind == Node::None, "fixture root is None");

    // A reducer naming a Python callable is recorded, never called.
    const std::string inert("\x80\x02" "cbuiltins\neval\n" ")R.");
    auto obj = mace::ckpt::unpickle(std::vector<char>(inert.begin(), inert.end()), zip);
    require(obj->kind == Node::Instance && obj->text == "builtins eval", "inert reducer");

    // Malformed pickles: memo miss, no STOP, SETITEMS without a mark, oversized string.
    require(rejects(std::string("\x80\x02" "h\x01.", 5), zip), "memo reference");
    require(rejects(std::string("\x80\x02" "N"), zip), "missing STOP");
    require(rejects(std::string("\x80\x02" "u."), zip), "SETITEMS without mark");
    require(rejects(std::string("\x80\x02" "X\xff\xff\xff\x7f.", 8), zip), "oversized string");
    require(rejects(std::string("\x80\x02" "NN.", 5), zip), "two values at STOP");
    require(rejects(std::string("\x80\x01" "N.", 4), zip), "protocol 1");
    require(rejects(std::string("\x80\x02" "I1\n.", 6), zip), "text opcode");

    // Views honour the storage offset and row strides, and stay inside the storage.
    mace::ckpt::Tensor t;
    t.dtype = "FloatStorage";
    const float storage[] = {0, 1, 2, 3, 4, 5};
    auto bytes = std::make_shared<std::vector<char>>(sizeof(storage));
    std::memcpy(bytes->data(), storage, sizeof(storage));
    t.storage = bytes;
    t.offset = 1;
    t.shape = {2, 2};
    t.stride = {3, 1};
    require(t.values() == std::vector<double>({1, 2, 4, 5}), "strided view");
    t.shape = {2, 2};
    t.stride = {1, 2};
    require(t.values() == std::vector<double>({1, 3, 2, 4}), "transposed view");
    t.offset = 2;
    t.stride = {3, 1};
    bool outside = false;
    try {
      t.values();
    } catch (const std::exception &) {
      outside = true;
    }
    require(outside, "view past the storage");
    std::cout << "ZIP fixture, inert reducers, malformed pickles and strided views passed\n";
  } catch (const std::exception &e) {
    std::cerr << e.what() << '\n';
    return 1;
  }
  return 0;
}
