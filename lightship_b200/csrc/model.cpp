// model.cpp -- ONNX models on the CUDA backend: the model loader, the graph optimizer's fusion
// decisions and an inference session, behind the C ABI (lsc_model_* / lsc_session_*).
//
//   loader     ONNX ModelProto bytes -> graph of nodes, initializers, inputs and outputs
//              (ModelLoader / OnnxLoader, lightship-core/src/model/onnx.rs).  Node attributes
//              are read (strides, pads, dilations, group, epsilon, transB, ...): the
//              reference's parser skips them (onnx.rs:613), so its Conv2d always runs with
//              stride 1 and no padding.
//   fusion     FusionPass (lightship-core/src/ir/optimizer.rs:505-890) with its single-consumer
//              rule (:633-640), applied in the order that reaches Conv+BN+ReLU: BatchNorm is
//              folded into its Conv first, then a following Relu / Clip(0, 6) becomes the
//              epilogue activation (the reference looks for Conv->Relu before Conv->BN and so
//              never fuses the ReLU of a Conv->BN->Relu chain); Add->Relu becomes AddReLU,
//              BatchNorm->Relu BatchNormReLU.
//   session    Engine::create_session / Session::run (LightShipEngine_CreateSession,
//              LightShipSession_Run, c-api/include/lightship.h:283-331): every node compiled
//              once through lsc_compile_operator with its initializers as weights, one device
//              buffer per intermediate tensor from the backend's arena, nodes executed in the
//              graph's (topological) order through lsc_execute on the caller's stream.
//
// The protobuf subset read here: ModelProto.graph (7); GraphProto node (1), name (2),
// initializer (5), input (11), output (12); NodeProto input (1), output (2), name (3),
// op_type (4), attribute (5); AttributeProto name (1), f (2), i (3), s (4), floats (7),
// ints (8); TensorProto dims (1), data_type (2), float_data (4), int32_data (5),
// int64_data (7), name (8), raw_data (9); ValueInfoProto name (1), type (2) -> tensor_type (1)
// -> elem_type (1), shape (2) -> dim (1) -> dim_value (1).
#include <math.h>
#include <string.h>

#include <map>
#include <memory>
#include <new>
#include <set>
#include <string>
#include <vector>

#include "backend_ops.h"

namespace {

using lsc::set_error;

// ------------------------------------------------------------------------------ protobuf
struct Reader {
  const uint8_t* p;
  const uint8_t* end;
  bool bad = false;

  bool more() const { return !bad && p < end; }
  uint64_t varint() {
    uint64_t v = 0;
    for (int shift = 0; shift < 64; shift += 7) {
      if (p >= end) {
        bad = true;
        return 0;
      }
      const uint8_t b = *p++;
      v |= static_cast<uint64_t>(b & 0x7F) << shift;
      if (!(b & 0x80)) return v;
    }
    bad = true;
    return 0;
  }
  uint32_t fixed32() {
    if (end - p < 4) {
      bad = true;
      return 0;
    }
    uint32_t v;
    memcpy(&v, p, 4);
    p += 4;
    return v;
  }
  Reader sub() {  // a length-delimited field's contents
    const uint64_t n = varint();
    if (bad || n > static_cast<uint64_t>(end - p)) {
      bad = true;
      return Reader{end, end, true};
    }
    Reader r{p, p + n};
    p += n;
    return r;
  }
  std::string str() {
    Reader r = sub();
    return std::string(reinterpret_cast<const char*>(r.p), static_cast<size_t>(r.end - r.p));
  }
  void skip(int wire) {
    switch (wire) {
      case 0: varint(); break;
      case 1:
        if (end - p < 8) bad = true; else p += 8;
        break;
      case 2: sub(); break;
      case 5: fixed32(); break;
      default: bad = true;
    }
  }
  // one key; false at the end or on a malformed key
  bool key(int& field, int& wire) {
    if (!more()) return false;
    const uint64_t k = varint();
    field = static_cast<int>(k >> 3);
    wire = static_cast<int>(k & 7);
    return !bad;
  }
};

float bits_to_float(uint32_t b) {
  float f;
  memcpy(&f, &b, 4);
  return f;
}

// a repeated scalar field, packed (wire 2) or not
void read_ints(Reader& r, int wire, std::vector<int64_t>& out) {
  if (wire == 2) {
    Reader s = r.sub();
    while (s.more()) out.push_back(static_cast<int64_t>(s.varint()));
    if (s.bad) r.bad = true;
  } else {
    out.push_back(static_cast<int64_t>(r.varint()));
  }
}
void read_floats(Reader& r, int wire, std::vector<float>& out) {
  if (wire == 2) {
    Reader s = r.sub();
    while (s.more()) out.push_back(bits_to_float(s.fixed32()));
    if (s.bad) r.bad = true;
  } else {
    out.push_back(bits_to_float(r.fixed32()));
  }
}

// ONNX TensorProto.DataType
constexpr int kOnnxFloat = 1, kOnnxInt32 = 6, kOnnxInt64 = 7;

struct OnnxTensor {
  std::string name;
  int data_type = 0;
  std::vector<int64_t> dims;
  std::vector<float> f;   // FLOAT data
  std::vector<int64_t> i; // INT32 / INT64 data
};

bool parse_tensor(Reader r, OnnxTensor& t) {
  std::string raw;
  int field, wire;
  while (r.key(field, wire)) {
    switch (field) {
      case 1: read_ints(r, wire, t.dims); break;
      case 2: t.data_type = static_cast<int>(r.varint()); break;
      case 4: read_floats(r, wire, t.f); break;
      case 5:
      case 7: read_ints(r, wire, t.i); break;
      case 8: t.name = r.str(); break;
      case 9: raw = r.str(); break;
      default: r.skip(wire);
    }
  }
  if (r.bad) return false;
  if (!raw.empty()) {
    if (t.data_type == kOnnxFloat) {
      t.f.resize(raw.size() / 4);
      memcpy(t.f.data(), raw.data(), t.f.size() * 4);
    } else if (t.data_type == kOnnxInt64) {
      t.i.resize(raw.size() / 8);
      memcpy(t.i.data(), raw.data(), t.i.size() * 8);
    } else if (t.data_type == kOnnxInt32) {
      std::vector<int32_t> v(raw.size() / 4);
      memcpy(v.data(), raw.data(), v.size() * 4);
      t.i.assign(v.begin(), v.end());
    }
  }
  // ONNX stores int32 data sign-extended in int64 varints; the varint read above is unsigned
  for (auto& v : t.i)
    if (t.data_type == kOnnxInt32) v = static_cast<int32_t>(static_cast<uint32_t>(v));
  return true;
}

struct OnnxAttr {
  std::string name;
  float f = 0.0f;
  int64_t i = 0;
  std::string s;
  std::vector<float> floats;
  std::vector<int64_t> ints;
};

bool parse_attr(Reader r, OnnxAttr& a) {
  int field, wire;
  while (r.key(field, wire)) {
    switch (field) {
      case 1: a.name = r.str(); break;
      case 2: a.f = bits_to_float(r.fixed32()); break;
      case 3: a.i = static_cast<int64_t>(r.varint()); break;
      case 4: a.s = r.str(); break;
      case 7: read_floats(r, wire, a.floats); break;
      case 8: read_ints(r, wire, a.ints); break;
      default: r.skip(wire);
    }
  }
  return !r.bad;
}

struct GraphIO {
  std::string name;
  int32_t dtype = LSC_DTYPE_F32;
  std::vector<int64_t> shape;  // -1 = symbolic
};

bool parse_value_info(Reader r, GraphIO& io) {
  int field, wire;
  while (r.key(field, wire)) {
    if (field == 1) {
      io.name = r.str();
    } else if (field == 2) {  // TypeProto
      Reader tp = r.sub();
      int f2, w2;
      while (tp.key(f2, w2)) {
        if (f2 != 1) {
          tp.skip(w2);
          continue;
        }
        Reader tt = tp.sub();  // TypeProto.Tensor
        int f3, w3;
        while (tt.key(f3, w3)) {
          if (f3 == 1) {
            const int et = static_cast<int>(tt.varint());
            io.dtype = et == kOnnxFloat ? LSC_DTYPE_F32 : et == kOnnxInt64 ? LSC_DTYPE_I64
                       : et == kOnnxInt32 ? LSC_DTYPE_I32 : -1;
          } else if (f3 == 2) {
            Reader shp = tt.sub();
            int f4, w4;
            while (shp.key(f4, w4)) {
              if (f4 != 1) {
                shp.skip(w4);
                continue;
              }
              Reader dim = shp.sub();
              int64_t v = -1;
              int f5, w5;
              while (dim.key(f5, w5)) {
                if (f5 == 1) v = static_cast<int64_t>(dim.varint());
                else dim.skip(w5);
              }
              if (dim.bad) shp.bad = true;
              io.shape.push_back(v);
            }
            if (shp.bad) tt.bad = true;
          } else {
            tt.skip(w3);
          }
        }
        if (tt.bad) tp.bad = true;
      }
      if (tp.bad) r.bad = true;
    } else {
      r.skip(wire);
    }
  }
  return !r.bad;
}

struct Node {
  std::string name, op;
  std::vector<std::string> in, out;
  std::vector<OnnxAttr> attrs;
  // after the fusion pass
  int32_t fusion = LSC_FUSION_NONE;
  int32_t activation = LSC_ACT_NONE;
  std::vector<std::string> bn;  // folded BatchNorm: gamma, beta, mean, var initializer names
  float bn_eps = 1e-5f;
  bool removed = false;

  const OnnxAttr* attr(const char* n) const {
    for (const auto& a : attrs)
      if (a.name == n) return &a;
    return nullptr;
  }
  int64_t attr_i(const char* n, int64_t dflt) const {
    const OnnxAttr* a = attr(n);
    return a ? a->i : dflt;
  }
  float attr_f(const char* n, float dflt) const {
    const OnnxAttr* a = attr(n);
    return a ? a->f : dflt;
  }
  std::vector<int64_t> attr_ints(const char* n) const {
    const OnnxAttr* a = attr(n);
    return a ? a->ints : std::vector<int64_t>();
  }
};

}  // namespace

struct lsc_model {
  std::string name;
  std::vector<Node> nodes;                  // fused graph, removed nodes erased
  std::map<std::string, OnnxTensor> inits;  // initializers by name
  std::vector<GraphIO> inputs, outputs;     // graph inputs that are not initializers; outputs
  std::vector<lsc_op_desc> descs;           // per node: the Backend operator it lowers to
};

namespace {

// how many nodes read tensor `t` (a graph output counts as one more reader)
int consumers(const lsc_model& m, const std::string& t) {
  int c = 0;
  for (const auto& n : m.nodes)
    if (!n.removed)
      for (const auto& i : n.in) c += (i == t);
  for (const auto& o : m.outputs) c += (o.name == t);
  return c;
}

Node* sole_consumer(lsc_model& m, const std::string& t) {
  if (consumers(m, t) != 1) return nullptr;
  for (auto& n : m.nodes)
    if (!n.removed)
      for (const auto& i : n.in)
        if (i == t) return &n;
  return nullptr;  // the one reader is a graph output
}

// Clip(min = 0, max = 6), from attributes (opset < 11) or constant inputs (opset >= 11)
bool is_relu6_clip(const lsc_model& m, const Node& n) {
  if (n.op != "Clip") return false;
  float lo = n.attr_f("min", -INFINITY), hi = n.attr_f("max", INFINITY);
  auto scalar = [&](size_t idx, float& v) {
    if (n.in.size() <= idx || n.in[idx].empty()) return;
    auto it = m.inits.find(n.in[idx]);
    if (it != m.inits.end() && it->second.f.size() == 1) v = it->second.f[0];
  };
  scalar(1, lo);
  scalar(2, hi);
  return lo == 0.0f && hi == 6.0f;
}

// `absorbed`'s output becomes `keeper`'s; `absorbed` leaves the graph
void absorb(Node& keeper, Node& absorbed) {
  keeper.out[0] = absorbed.out[0];
  absorbed.removed = true;
}

void fusion_pass(lsc_model& m) {
  for (auto& n : m.nodes) {
    if (n.removed || n.out.empty()) continue;
    if (n.op == "Conv") {
      Node* c = sole_consumer(m, n.out[0]);
      if (c && c->op == "BatchNormalization" && c->in.size() >= 5 && c->in[0] == n.out[0]) {
        n.fusion = LSC_FUSION_CONV_BATCHNORM;
        n.bn = {c->in[1], c->in[2], c->in[3], c->in[4]};
        n.bn_eps = c->attr_f("epsilon", 1e-5f);
        absorb(n, *c);
        c = sole_consumer(m, n.out[0]);
      }
      if (c && (c->op == "Relu" || is_relu6_clip(m, *c))) {
        const bool six = c->op != "Relu";
        if (n.fusion == LSC_FUSION_NONE) n.fusion = six ? LSC_FUSION_CONV_RELU6 : LSC_FUSION_CONV_RELU;
        else n.activation = six ? LSC_ACT_RELU6 : LSC_ACT_RELU;
        absorb(n, *c);
      }
    } else if (n.op == "Add" || n.op == "BatchNormalization") {
      Node* c = sole_consumer(m, n.out[0]);
      if (c && c->op == "Relu") {
        n.fusion = n.op == "Add" ? LSC_FUSION_ADD_RELU : LSC_FUSION_BATCHNORM_RELU;
        absorb(n, *c);
      }
    }
  }
  std::vector<Node> kept;
  for (auto& n : m.nodes)
    if (!n.removed) kept.push_back(std::move(n));
  m.nodes.swap(kept);
}

lsc_op_desc base_desc(int32_t op_type) {
  lsc_op_desc d{};
  d.op_type = op_type;
  d.fusion = LSC_FUSION_NONE;
  d.stride_h = d.stride_w = 1;
  d.dilation_h = d.dilation_w = 1;
  d.groups = 1;
  d.rounding = -1;
  d.fp32_mode = -1;
  return d;
}

// Node -> Backend operator descriptor; op_type -1 = a view (Flatten / Reshape: no kernel)
lsc_status lower(const lsc_model& m, const Node& n, lsc_op_desc& d) {
  const std::string& op = n.op;
  if (op == "Conv" || op == "MaxPool") {
    d = base_desc(op == "Conv" ? LSC_OP_CONV2D : LSC_OP_MAXPOOL2D);
    const auto strides = n.attr_ints("strides"), pads = n.attr_ints("pads"), dil = n.attr_ints("dilations");
    if (!n.attr_ints("kernel_shape").empty() && n.attr_ints("kernel_shape").size() != 2)
      return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "node '%s': only 2-D %s", n.name.c_str(), op.c_str());
    if (strides.size() == 2) {
      d.stride_h = static_cast<int32_t>(strides[0]);
      d.stride_w = static_cast<int32_t>(strides[1]);
    }
    if (dil.size() == 2) {
      d.dilation_h = static_cast<int32_t>(dil[0]);
      d.dilation_w = static_cast<int32_t>(dil[1]);
    }
    if (pads.size() == 4) {  // [top, left, bottom, right]
      d.pad_h = static_cast<int32_t>(pads[0]);
      d.pad_w = static_cast<int32_t>(pads[1]);
      d.pad_h_end_delta = static_cast<int32_t>(pads[2] - pads[0]);
      d.pad_w_end_delta = static_cast<int32_t>(pads[3] - pads[1]);
    }
    const OnnxAttr* ap = n.attr("auto_pad");
    if (ap && !ap->s.empty() && ap->s != "NOTSET")
      return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "node '%s': auto_pad %s", n.name.c_str(), ap->s.c_str());
    if (op == "Conv") {
      d.groups = static_cast<int32_t>(n.attr_i("group", 1));
      d.fusion = n.fusion;
      d.activation = n.activation;
      d.bn_epsilon = n.bn_eps;
    } else {
      const auto ks = n.attr_ints("kernel_shape");
      if (ks.size() != 2) return set_error(LSC_ERROR_INVALID_ARGUMENT, "node '%s': MaxPool without kernel_shape", n.name.c_str());
      d.kernel_h = static_cast<int32_t>(ks[0]);
      d.kernel_w = static_cast<int32_t>(ks[1]);
      if (d.pad_h_end_delta || d.pad_w_end_delta || n.attr_i("ceil_mode", 0))
        return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "node '%s': MaxPool with asymmetric padding or ceil_mode",
                         n.name.c_str());
    }
    return LSC_SUCCESS;
  }
  if (op == "BatchNormalization") {
    d = base_desc(LSC_OP_BATCHNORM);
    d.fusion = n.fusion;
    d.bn_epsilon = n.attr_f("epsilon", 1e-5f);
    return LSC_SUCCESS;
  }
  if (op == "Relu" || is_relu6_clip(m, n)) {
    d = base_desc(op == "Relu" ? LSC_OP_RELU : LSC_OP_RELU6);
    return LSC_SUCCESS;
  }
  if (op == "Add") {
    d = base_desc(LSC_OP_ADD);
    d.fusion = n.fusion;
    return LSC_SUCCESS;
  }
  if (op == "GlobalAveragePool") {
    d = base_desc(LSC_OP_GLOBAL_AVGPOOL2D);
    return LSC_SUCCESS;
  }
  if (op == "Gemm" || op == "MatMul") {
    if (op == "Gemm" && (n.attr_i("transA", 0) != 0 || n.attr_f("alpha", 1.0f) != 1.0f || n.attr_f("beta", 1.0f) != 1.0f))
      return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "node '%s': Gemm with transA or alpha/beta != 1", n.name.c_str());
    // a constant right operand becomes FullyConnected's [N, K] weight; else a runtime MatMul
    d = base_desc(n.in.size() > 1 && m.inits.count(n.in[1]) ? LSC_OP_FULLY_CONNECTED : LSC_OP_MATMUL);
    if (d.op_type == LSC_OP_MATMUL && (op == "Gemm" && (n.attr_i("transB", 0) != 0 || n.in.size() > 2)))
      return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "node '%s': Gemm with a runtime B needs transB = 0 and no C",
                       n.name.c_str());
    return LSC_SUCCESS;
  }
  if (op == "Softmax") {
    d = base_desc(LSC_OP_SOFTMAX);
    return LSC_SUCCESS;
  }
  if (op == "LayerNormalization") {
    d = base_desc(LSC_OP_LAYERNORM);
    d.bn_epsilon = n.attr_f("epsilon", 1e-5f);
    return LSC_SUCCESS;
  }
  if (op == "Gelu") {
    d = base_desc(LSC_OP_GELU);
    return LSC_SUCCESS;
  }
  if (op == "Flatten" || op == "Reshape") {
    d = base_desc(-1);
    return LSC_SUCCESS;
  }
  return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "node '%s': ONNX operator %s is not supported by the CUDA backend",
                   n.name.c_str(), op.c_str());
}

lsc_status parse_model(const uint8_t* data, uint64_t size, lsc_model& m) {
  Reader r{data, data + size};
  int field, wire;
  bool have_graph = false;
  while (r.key(field, wire)) {
    if (field != 7 || wire != 2) {
      r.skip(wire);
      continue;
    }
    have_graph = true;
    Reader g = r.sub();
    std::vector<GraphIO> declared;
    int gf, gw;
    while (g.key(gf, gw)) {
      if (gf == 1) {
        Reader nr = g.sub();
        Node n;
        int nf, nw;
        while (nr.key(nf, nw)) {
          switch (nf) {
            case 1: n.in.push_back(nr.str()); break;
            case 2: n.out.push_back(nr.str()); break;
            case 3: n.name = nr.str(); break;
            case 4: n.op = nr.str(); break;
            case 5: {
              OnnxAttr a;
              if (!parse_attr(nr.sub(), a)) nr.bad = true;
              n.attrs.push_back(std::move(a));
              break;
            }
            default: nr.skip(nw);
          }
        }
        if (nr.bad) g.bad = true;
        if (n.name.empty()) n.name = n.op + "_" + std::to_string(m.nodes.size());
        m.nodes.push_back(std::move(n));
      } else if (gf == 2) {
        m.name = g.str();
      } else if (gf == 5) {
        OnnxTensor t;
        if (!parse_tensor(g.sub(), t)) g.bad = true;
        m.inits[t.name] = std::move(t);
      } else if (gf == 11 || gf == 12) {
        GraphIO io;
        if (!parse_value_info(g.sub(), io)) g.bad = true;
        (gf == 11 ? declared : m.outputs).push_back(std::move(io));
      } else {
        g.skip(gw);
      }
    }
    if (g.bad) r.bad = true;
    for (auto& io : declared)
      if (!m.inits.count(io.name)) m.inputs.push_back(std::move(io));
  }
  if (r.bad) return set_error(LSC_ERROR_INVALID_ARGUMENT, "ONNX model: malformed protobuf");
  if (!have_graph || m.nodes.empty()) return set_error(LSC_ERROR_INVALID_ARGUMENT, "ONNX model: no graph");
  for (const auto& n : m.nodes)
    if (n.out.empty() || n.in.empty())
      return set_error(LSC_ERROR_INVALID_ARGUMENT, "ONNX model: node '%s' without inputs or outputs", n.name.c_str());
  return LSC_SUCCESS;
}

}  // namespace

// ------------------------------------------------------------------------------ session
namespace {

struct Value {
  std::vector<int64_t> shape;
  void* dev = nullptr;      // arena buffer (intermediates) or nullptr (bound at run)
  int alias_of = -1;        // a view of another value (Flatten / Reshape)
  int input_index = -1;     // graph input position
  int output_index = -1;    // graph output position
};

int64_t count_of(const std::vector<int64_t>& s) {
  int64_t c = 1;
  for (auto v : s) c *= v;
  return c;
}

lsc_tensor host_f32(const char* name, const std::vector<int64_t>& shape, const float* data) {
  lsc_tensor t{};
  t.name = name;
  t.ndim = static_cast<int32_t>(shape.size());
  for (size_t i = 0; i < shape.size(); ++i) t.shape[i] = shape[i];
  t.dtype = LSC_DTYPE_F32;
  t.layout = LSC_LAYOUT_DEFAULT;
  t.location = LSC_MEM_HOST;
  t.data = const_cast<float*>(data);
  t.nbytes = static_cast<uint64_t>(count_of(shape)) * 4;
  return t;
}

}  // namespace

struct lsc_session {
  lsc_backend* be = nullptr;
  const lsc_model* model = nullptr;
  std::map<std::string, int> ids;
  std::vector<Value> values;
  struct Step {
    lsc_op* op = nullptr;               // nullptr for a view
    std::vector<int> in, out;           // value ids read / written at run time
  };
  std::vector<Step> steps;
  std::vector<lsc_memory_block> blocks;
  ~lsc_session() {
    for (auto& s : steps)
      if (s.op) lsc_op_destroy(s.op);
    for (auto& b : blocks) lsc_deallocate(be, &b);
    if (be) be->release();
  }
};

namespace {

// output shape of a lowered node from its input shapes (NCHW)
lsc_status infer_shape(const lsc_model& m, const Node& n, const lsc_op_desc& d,
                       const std::vector<std::vector<int64_t>>& in, std::vector<int64_t>& out) {
  const auto& x = in[0];
  auto need4 = [&]() -> lsc_status {
    if (x.size() != 4) return set_error(LSC_ERROR_SHAPE_MISMATCH, "node '%s': needs a 4-D NCHW input", n.name.c_str());
    return LSC_SUCCESS;
  };
  lsc_status st;
  switch (d.op_type) {
    case LSC_OP_CONV2D: {
      if ((st = need4())) return st;
      const OnnxTensor& w = m.inits.at(n.in[1]);
      if (w.dims.size() != 4) return set_error(LSC_ERROR_SHAPE_MISMATCH, "node '%s': 4-D filter expected", n.name.c_str());
      const int64_t kh = w.dims[2], kw = w.dims[3];
      const int64_t oh = (x[2] + 2 * d.pad_h + d.pad_h_end_delta - d.dilation_h * (kh - 1) - 1) / d.stride_h + 1;
      const int64_t ow = (x[3] + 2 * d.pad_w + d.pad_w_end_delta - d.dilation_w * (kw - 1) - 1) / d.stride_w + 1;
      out = {x[0], w.dims[0], oh, ow};
      return LSC_SUCCESS;
    }
    case LSC_OP_MAXPOOL2D: {
      if ((st = need4())) return st;
      out = {x[0], x[1], (x[2] + 2 * d.pad_h - d.kernel_h) / d.stride_h + 1,
             (x[3] + 2 * d.pad_w - d.kernel_w) / d.stride_w + 1};
      return LSC_SUCCESS;
    }
    case LSC_OP_GLOBAL_AVGPOOL2D:
      if ((st = need4())) return st;
      out = {x[0], x[1], 1, 1};
      return LSC_SUCCESS;
    case LSC_OP_FULLY_CONNECTED: {
      const OnnxTensor& w = m.inits.at(n.in[1]);
      const bool trans_b = n.op == "Gemm" && n.attr_i("transB", 0) != 0;
      if (w.dims.size() != 2 || x.size() != 2)
        return set_error(LSC_ERROR_SHAPE_MISMATCH, "node '%s': 2-D operands expected", n.name.c_str());
      out = {x[0], trans_b ? w.dims[0] : w.dims[1]};
      return LSC_SUCCESS;
    }
    case LSC_OP_MATMUL:
      if (x.size() != 2 || in[1].size() != 2)
        return set_error(LSC_ERROR_SHAPE_MISMATCH, "node '%s': 2-D operands expected", n.name.c_str());
      out = {x[0], in[1][1]};
      return LSC_SUCCESS;
    case -1: {  // Flatten (axis) / Reshape (constant shape)
      if (n.op == "Flatten") {
        int64_t axis = n.attr_i("axis", 1);
        if (axis < 0) axis += static_cast<int64_t>(x.size());
        int64_t a = 1, b = 1;
        for (size_t i = 0; i < x.size(); ++i) (static_cast<int64_t>(i) < axis ? a : b) *= x[i];
        out = {a, b};
        return LSC_SUCCESS;
      }
      auto it = n.in.size() > 1 ? m.inits.find(n.in[1]) : m.inits.end();
      if (it == m.inits.end()) return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "node '%s': Reshape needs a constant shape", n.name.c_str());
      out = it->second.i;
      int64_t known = 1, infer = -1;
      for (size_t i = 0; i < out.size(); ++i) {
        if (out[i] == 0 && i < x.size()) out[i] = x[i];
        if (out[i] == -1) infer = static_cast<int64_t>(i);
        else known *= out[i];
      }
      if (infer >= 0) out[static_cast<size_t>(infer)] = known ? count_of(x) / known : 0;
      if (count_of(out) != count_of(x))
        return set_error(LSC_ERROR_SHAPE_MISMATCH, "node '%s': Reshape changes the element count", n.name.c_str());
      return LSC_SUCCESS;
    }
    default:  // elementwise / row-wise: the input's shape
      out = x;
      return LSC_SUCCESS;
  }
}

lsc_status build_session(lsc_session& s, const lsc_model& m) {
  auto value_of = [&](const std::string& name) -> int {
    auto it = s.ids.find(name);
    if (it != s.ids.end()) return it->second;
    s.values.emplace_back();
    s.ids[name] = static_cast<int>(s.values.size()) - 1;
    return static_cast<int>(s.values.size()) - 1;
  };
  for (size_t i = 0; i < m.inputs.size(); ++i) {
    const auto& io = m.inputs[i];
    for (auto v : io.shape)
      if (v <= 0)
        return set_error(LSC_ERROR_SHAPE_MISMATCH, "graph input '%s' has a symbolic or empty dimension", io.name.c_str());
    if (io.dtype != LSC_DTYPE_F32)
      return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "graph input '%s' is not f32", io.name.c_str());
    const int id = value_of(io.name);
    s.values[id].shape = io.shape;
    s.values[id].input_index = static_cast<int>(i);
  }
  for (size_t i = 0; i < m.outputs.size(); ++i) {
    const int id = value_of(m.outputs[i].name);
    s.values[id].output_index = static_cast<int>(i);
  }
  for (size_t k = 0; k < m.nodes.size(); ++k) {
    const Node& n = m.nodes[k];
    const lsc_op_desc& d = m.descs[k];
    lsc_session::Step step;
    std::vector<std::vector<int64_t>> in_shapes;
    // activations: inputs that are not initializers
    for (const auto& t : n.in) {
      if (t.empty() || m.inits.count(t)) continue;
      auto it = s.ids.find(t);
      if (it == s.ids.end() || s.values[it->second].shape.empty())
        return set_error(LSC_ERROR_INVALID_ARGUMENT, "node '%s': input '%s' is produced by no earlier node",
                         n.name.c_str(), t.c_str());
      step.in.push_back(it->second);
      in_shapes.push_back(s.values[it->second].shape);
    }
    if (in_shapes.empty())
      return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "node '%s': no runtime input", n.name.c_str());
    if ((d.op_type == LSC_OP_ADD || d.op_type == LSC_OP_MATMUL) && step.in.size() != 2)
      return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "node '%s': %s of a constant operand is not supported",
                       n.name.c_str(), n.op.c_str());
    std::vector<int64_t> oshape;
    lsc_status st = infer_shape(m, n, d, in_shapes, oshape);
    if (st) return st;
    const int oid = value_of(n.out[0]);
    s.values[oid].shape = oshape;
    step.out.push_back(oid);
    if (d.op_type == -1) {
      s.values[oid].alias_of = step.in[0];
      s.steps.push_back(step);
      continue;
    }
    // compile with the initializers as weights (host tensors), activations as shape-only
    std::vector<lsc_tensor> cin;
    std::vector<std::vector<float>> tmp;  // Gemm B transposed / MatMul B as [N, K]
    tmp.reserve(2);
    size_t act_i = 0;
    for (const auto& t : n.in) {
      if (t.empty()) {
        cin.push_back(lsc_tensor{});
        continue;
      }
      auto it = m.inits.find(t);
      if (it == m.inits.end()) {
        lsc_tensor a{};
        a.name = t.c_str();
        const auto& shp = in_shapes[act_i++];
        a.ndim = static_cast<int32_t>(shp.size());
        for (size_t i = 0; i < shp.size(); ++i) a.shape[i] = shp[i];
        a.dtype = LSC_DTYPE_F32;
        a.layout = LSC_LAYOUT_NCHW;
        a.location = LSC_MEM_DEVICE;
        cin.push_back(a);
        continue;
      }
      const OnnxTensor& w = it->second;
      if (w.data_type != kOnnxFloat || static_cast<int64_t>(w.f.size()) != count_of(w.dims))
        return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "initializer '%s' must be f32 with its data", t.c_str());
      const bool weight_kn = d.op_type == LSC_OP_FULLY_CONNECTED && &t == &n.in[1] &&
                             !(n.op == "Gemm" && n.attr_i("transB", 0) != 0);
      if (weight_kn) {  // [K, N] -> FullyConnected's [N, K]
        const int64_t kk = w.dims[0], nn = w.dims[1];
        tmp.emplace_back(static_cast<size_t>(kk * nn));
        for (int64_t a = 0; a < kk; ++a)
          for (int64_t b = 0; b < nn; ++b) tmp.back()[b * kk + a] = w.f[a * nn + b];
        cin.push_back(host_f32(t.c_str(), {nn, kk}, tmp.back().data()));
      } else {
        cin.push_back(host_f32(t.c_str(), w.dims, w.f.data()));
      }
    }
    for (const auto& b : n.bn) {  // folded BatchNorm parameters follow X, W, B
      auto it = m.inits.find(b);
      if (it == m.inits.end()) return set_error(LSC_ERROR_INVALID_ARGUMENT, "node '%s': BatchNorm parameter '%s' is not constant", n.name.c_str(), b.c_str());
      while (cin.size() < 3) cin.push_back(lsc_tensor{});
      cin.push_back(host_f32(b.c_str(), it->second.dims, it->second.f.data()));
    }
    lsc_tensor cout_t{};
    cout_t.name = n.out[0].c_str();
    cout_t.ndim = static_cast<int32_t>(oshape.size());
    for (size_t i = 0; i < oshape.size(); ++i) cout_t.shape[i] = oshape[i];
    cout_t.dtype = LSC_DTYPE_F32;
    cout_t.location = LSC_MEM_DEVICE;
    st = lsc_compile_operator(s.be, &d, cin.data(), static_cast<int32_t>(cin.size()), &cout_t, 1, &step.op);
    if (st) return st;
    s.steps.push_back(step);
  }
  for (size_t i = 0; i < m.outputs.size(); ++i)
    if (s.values[s.ids[m.outputs[i].name]].shape.empty())
      return set_error(LSC_ERROR_INVALID_ARGUMENT, "graph output '%s' is produced by no node", m.outputs[i].name.c_str());
  // device buffers for intermediates (graph inputs and outputs are the caller's)
  for (auto& v : s.values) {
    if (v.input_index >= 0 || v.output_index >= 0 || v.alias_of >= 0 || v.shape.empty()) continue;
    lsc_memory_block b{};
    lsc_status st = lsc_allocate(s.be, static_cast<uint64_t>(count_of(v.shape)) * 4, 256, &b);
    if (st) return st;
    s.blocks.push_back(b);
    v.dev = b.ptr;
  }
  return LSC_SUCCESS;
}

}  // namespace

// ------------------------------------------------------------------------------ C ABI
extern "C" {

lsc_status lsc_model_load_onnx(const uint8_t* data, uint64_t size, lsc_model** out) {
  if (!out) return set_error(LSC_ERROR_INVALID_ARGUMENT, "lsc_model_load_onnx: null output");
  *out = nullptr;
  if (!data || size == 0) return set_error(LSC_ERROR_INVALID_ARGUMENT, "lsc_model_load_onnx: empty model");
  std::unique_ptr<lsc_model> m(new (std::nothrow) lsc_model());
  if (!m) return set_error(LSC_ERROR_OUT_OF_MEMORY, "lsc_model_load_onnx: out of host memory");
  lsc_status st = parse_model(data, size, *m);
  if (st) return st;
  fusion_pass(*m);
  m->descs.resize(m->nodes.size());
  for (size_t i = 0; i < m->nodes.size(); ++i)
    if ((st = lower(*m, m->nodes[i], m->descs[i]))) return st;
  *out = m.release();
  return LSC_SUCCESS;
}

void lsc_model_destroy(lsc_model* model) { delete model; }

lsc_status lsc_model_info(const lsc_model* model, uint32_t* n_inputs, uint32_t* n_outputs, uint32_t* n_nodes) {
  if (!model) return set_error(LSC_ERROR_INVALID_ARGUMENT, "lsc_model_info: null model");
  if (n_inputs) *n_inputs = static_cast<uint32_t>(model->inputs.size());
  if (n_outputs) *n_outputs = static_cast<uint32_t>(model->outputs.size());
  if (n_nodes) *n_nodes = static_cast<uint32_t>(model->nodes.size());
  return LSC_SUCCESS;
}

lsc_status lsc_model_io(const lsc_model* model, int32_t is_output, uint32_t index, const char** name,
                        int32_t* dtype, int64_t* shape, uint32_t* ndim) {
  if (!model) return set_error(LSC_ERROR_INVALID_ARGUMENT, "lsc_model_io: null model");
  const auto& v = is_output ? model->outputs : model->inputs;
  if (index >= v.size()) return set_error(LSC_ERROR_INVALID_ARGUMENT, "lsc_model_io: index %u out of range", index);
  const GraphIO& io = v[index];
  if (name) *name = io.name.c_str();
  if (dtype) *dtype = io.dtype;
  if (ndim) *ndim = static_cast<uint32_t>(io.shape.size());
  if (shape)
    for (size_t i = 0; i < io.shape.size() && i < LSC_MAX_DIMS; ++i) shape[i] = io.shape[i];
  return LSC_SUCCESS;
}

lsc_status lsc_model_node(const lsc_model* model, uint32_t index, lsc_op_desc* desc, const char** name,
                          const char** onnx_op) {
  if (!model) return set_error(LSC_ERROR_INVALID_ARGUMENT, "lsc_model_node: null model");
  if (index >= model->nodes.size()) return set_error(LSC_ERROR_INVALID_ARGUMENT, "lsc_model_node: index out of range");
  if (desc) *desc = model->descs[index];
  if (name) *name = model->nodes[index].name.c_str();
  if (onnx_op) *onnx_op = model->nodes[index].op.c_str();
  return LSC_SUCCESS;
}

lsc_status lsc_session_create(lsc_backend* backend, const lsc_model* model, lsc_session** out) {
  if (!backend || !model || !out) return set_error(LSC_ERROR_INVALID_ARGUMENT, "lsc_session_create: null argument");
  *out = nullptr;
  lsc::DeviceGuard guard(backend->device);
  if (!guard.ok()) return LSC_ERROR_DEVICE_ERROR;
  std::unique_ptr<lsc_session> s(new (std::nothrow) lsc_session());
  if (!s) return set_error(LSC_ERROR_OUT_OF_MEMORY, "lsc_session_create: out of host memory");
  backend->retain();
  s->be = backend;
  s->model = model;
  lsc_status st = build_session(*s, *model);
  if (st) return st;
  *out = s.release();
  return LSC_SUCCESS;
}

void lsc_session_destroy(lsc_session* session) { delete session; }

lsc_status lsc_session_run(lsc_session* s, const lsc_tensor* inputs, uint32_t n_inputs, lsc_tensor* outputs,
                           uint32_t n_outputs, lsc_stream stream) {
  if (!s) return set_error(LSC_ERROR_INVALID_ARGUMENT, "lsc_session_run: null session");
  const lsc_model& m = *s->model;
  if (n_inputs != m.inputs.size() || n_outputs != m.outputs.size() || (n_inputs && !inputs) || (n_outputs && !outputs))
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "lsc_session_run: the model takes %zu inputs and %zu outputs",
                     m.inputs.size(), m.outputs.size());
  for (uint32_t i = 0; i < n_inputs; ++i) {
    const auto& want = s->values[s->ids.at(m.inputs[i].name)].shape;
    const lsc_tensor& t = inputs[i];
    bool ok = t.dtype == LSC_DTYPE_F32 && t.ndim == static_cast<int32_t>(want.size()) && t.data;
    for (size_t d = 0; ok && d < want.size(); ++d) ok = t.shape[d] == want[d];
    if (!ok) return set_error(LSC_ERROR_SHAPE_MISMATCH, "lsc_session_run: input %u must be f32 of the model's shape", i);
  }
  // the tensor each value is read from / written to
  auto tensor_of = [&](int id, lsc_tensor& t) -> const lsc_tensor* {
    int base = id;
    while (s->values[base].alias_of >= 0) base = s->values[base].alias_of;
    const Value& v = s->values[base];
    const lsc_tensor* user = v.input_index >= 0 ? &inputs[v.input_index]
                             : v.output_index >= 0 ? &outputs[v.output_index] : nullptr;
    if (user) {
      t = *user;
    } else {
      t = lsc_tensor{};
      t.dtype = LSC_DTYPE_F32;
      t.location = LSC_MEM_DEVICE;
      t.data = v.dev;
      t.nbytes = static_cast<uint64_t>(count_of(v.shape)) * 4;
    }
    const auto& shp = s->values[id].shape;  // the view's own shape
    t.ndim = static_cast<int32_t>(shp.size());
    for (size_t i = 0; i < shp.size(); ++i) t.shape[i] = shp[i];
    t.layout = LSC_LAYOUT_NCHW;
    return user;
  };
  for (size_t k = 0; k < s->steps.size(); ++k) {
    const auto& step = s->steps[k];
    if (!step.op) {
      // a view: a graph output that is a view of an intermediate needs the data copied out
      const Value& v = s->values[step.out[0]];
      if (v.output_index >= 0) {
        lsc_tensor src{}, dst{};
        tensor_of(step.in[0], src);
        tensor_of(step.out[0], dst);
        if (dst.location == LSC_MEM_HOST) {
          lsc_status st = lsc_memcpy_d2h(dst.data, src.data, src.nbytes, stream);
          if (st) return st;
        } else if (cudaMemcpyAsync(dst.data, src.data, src.nbytes, cudaMemcpyDeviceToDevice,
                                   static_cast<cudaStream_t>(stream)) != cudaSuccess) {
          return set_error(LSC_ERROR_DEVICE_ERROR, "lsc_session_run: device copy failed");
        }
      }
      continue;
    }
    std::vector<lsc_tensor> in(step.in.size()), out(1);
    for (size_t i = 0; i < step.in.size(); ++i) tensor_of(step.in[i], in[i]);
    tensor_of(step.out[0], out[0]);
    lsc_status st = lsc_execute(s->be, step.op, in.data(), static_cast<int32_t>(in.size()), out.data(), 1, stream);
    if (st) return st;
    const Value& v = s->values[step.out[0]];
    if (v.output_index >= 0) {  // report the shape the backend produced
      lsc_tensor& o = outputs[v.output_index];
      o.ndim = out[0].ndim;
      for (int i = 0; i < o.ndim; ++i) o.shape[i] = out[0].shape[i];
    }
  }
  return LSC_SUCCESS;
}

}  // extern "C"
