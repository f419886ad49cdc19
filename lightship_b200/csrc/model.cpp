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

#include <algorithm>
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

struct QSession;                      // the INT8 session (below)
void destroy_qsession(QSession* q);

struct lsc_session {
  lsc_backend* be = nullptr;
  const lsc_model* model = nullptr;
  QSession* q = nullptr;               // set for INT8 sessions
  std::map<std::string, int> ids;
  std::vector<Value> values;
  struct Step {
    lsc_op* op = nullptr;               // nullptr for a view
    std::vector<int> in, out;           // value ids read / written at run time
  };
  std::vector<Step> steps;
  std::vector<lsc_memory_block> blocks;
  ~lsc_session() {
    destroy_qsession(q);
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

// ------------------------------------------------------------------------------ INT8 session
// An ONNX CNN compiled into the INT8 chain (Engine::create_session with a quantized backend):
//   lowering      Conv (+ folded BatchNorm, + ReLU / ReLU6) -> INT8 NHWC convolution with the
//                 filter quantized per output channel; an Add (+ ReLU) whose one operand is a
//                 convolution read by nothing else -> that convolution's fused residual
//                 (FusionType::AddReLU, ir/fusion.rs:20); MaxPool -> int8 max pool (the max
//                 commutes with the positive per-tensor scale); GlobalAveragePool -> int8
//                 average pool; Flatten / Reshape -> views; Gemm / MatMul with a constant
//                 weight -> INT8 FullyConnected with f32 output (the model's output).  The f32
//                 NCHW graph input is quantized to int8 NHWC (channels stored as a multiple of
//                 16); a first convolution of stride 2 over at most 4 channels runs as the
//                 stride-1 convolution of the space-to-depth input (2 x 2 pixel blocks folded
//                 into channels, the width rounded up to a multiple of 4 so it can run
//                 pixel-grouped), which sums the same products.
//   calibration   per-tensor symmetric scales (find_scale_zp, quantization/helpers.rs:101-136)
//                 of the input and of every layer's dequantized f32 output on a calibration
//                 batch, layer by layer, each layer then run again with its int8 output.
//   memory plan   every int8 activation gets an offset in one arena block: values whose
//                 live ranges (first write .. last read, in schedule order) overlap never share
//                 bytes; largest first, lowest fitting offset (the reference's MemoryPlan,
//                 executor/plan.rs:67-118, computes no offsets: scheduler.rs:196-226).
//   schedule      node order, with a convolution that reads the same tensor as the one before
//                 it (a ResNet block's downsample beside its first convolution) on a second
//                 stream; its consumer waits for it (GraphExecutor::execute_parallel,
//                 executor/graph_executor.rs:240-320, runs independent nodes concurrently).
//   run           the schedule captured once as a CUDA graph per input slot (two slots, so
//                 step i+1's input upload can overlap step i in lsc_session_run_async); the
//                 kernels keep their programmatic dependent launches inside the graph.
namespace {

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

struct QVal {
  std::string name;
  int64_t n = 0, h = 0, w = 0, c = 0;  // logical NHWC (c = the model's channels)
  int64_t w_store = 0, c_store = 0;    // stored width / channels
  float scale = 1.0f;
  bool flat = false;                   // [n, c] (pooled / flattened)
  int64_t offset = -1;                 // in the activation block
  int def = -1, last = -1;             // schedule positions
  int64_t bytes() const { return flat ? n * c_store : n * h * w_store * c_store; }
};

struct QStep {
  enum Kind { kInput, kConv, kMaxPool, kAvgPool, kFc } kind = kConv;
  int node = -1;           // model node index (the conv / pool / fc)
  int in = -1, res = -1, out = -1;
  int act = LSC_ACT_NONE;  // conv activation (after the residual)
  bool side = false;       // runs on the second stream beside the step before it
  int pos = 0;             // schedule position (liveness)
  lsc_op* op = nullptr;
  // max pool window (kernel, stride, padding), square
  int pool_k = 0, pool_s = 0, pool_p = 0;
  // stem (space-to-depth) geometry
  bool s2d = false;
  int64_t s2d_pad = 0, s2d_extra = 0;
};

}  // namespace

struct QSession {
  lsc_backend* be = nullptr;
  int rounding = LSC_ROUND_HALF_AWAY;
  bool concurrent = true;
  bool plan_memory = true;
  std::vector<QVal> vals;
  std::vector<QStep> steps;
  std::map<std::string, int> val_of;  // tensor name -> value id
  std::vector<int64_t> in_shape;      // f32 NCHW
  int64_t out_classes = 0;
  float in_scale = 1.0f;
  void* in_slot[2] = {nullptr, nullptr};
  void* out_buf = nullptr;
  void* act_block = nullptr;       // planned activations (plan_memory) ...
  std::vector<void*> act_blocks;   // ... or one block per value
  uint64_t planned_bytes = 0, unplanned_bytes = 0;
  cudaStream_t cap_stream = nullptr, side_stream = nullptr, copy_stream = nullptr;
  std::vector<cudaEvent_t> fork_ev, join_ev;
  cudaEvent_t slot_loaded[2] = {nullptr, nullptr}, slot_free[2] = {nullptr, nullptr};
  cudaGraphExec_t exec[2] = {nullptr, nullptr};
  int next_slot = 0;
  // the stem (input quantize, 7x7 / 2 convolution, 3x3 / 2 max pool) as one launch
  // (lsc::launch_stem_conv_pool_i8) with its filter image
  bool stem_fused = false;
  void* stem_w = nullptr;
  ~QSession() {
    for (auto& e : exec)
      if (e) cudaGraphExecDestroy(e);
    for (auto e : fork_ev) cudaEventDestroy(e);
    for (auto e : join_ev) cudaEventDestroy(e);
    for (int k = 0; k < 2; ++k) {
      if (slot_loaded[k]) cudaEventDestroy(slot_loaded[k]);
      if (slot_free[k]) cudaEventDestroy(slot_free[k]);
    }
    if (cap_stream) cudaStreamDestroy(cap_stream);
    if (side_stream) cudaStreamDestroy(side_stream);
    if (copy_stream) cudaStreamDestroy(copy_stream);
    for (auto& s : steps)
      if (s.op) lsc_op_destroy(s.op);
    if (be) {
      for (void* p : {in_slot[0], in_slot[1], out_buf, act_block, stem_w})
        if (p) be->arena.free(p);
      for (void* p : act_blocks) be->arena.free(p);
    }
  }
  void* ptr(int v) const {
    return plan_memory ? static_cast<char*>(act_block) + vals[v].offset : act_blocks[v];
  }
};

namespace {

lsc_tensor q_tensor(const QVal& v, void* data, float* scale_slot) {
  lsc_tensor t{};
  t.name = v.name.c_str();
  if (v.flat) {
    t.ndim = 2;
    t.shape[0] = v.n;
    t.shape[1] = v.c_store;
  } else {
    t.ndim = 4;
    t.shape[0] = v.n;
    t.shape[1] = v.h;
    t.shape[2] = v.w_store;
    t.shape[3] = v.c_store;
  }
  t.dtype = LSC_DTYPE_QINT8;
  t.layout = LSC_LAYOUT_NHWC;
  t.location = LSC_MEM_DEVICE;
  t.data = data;
  t.nbytes = static_cast<uint64_t>(v.bytes());
  *scale_slot = v.scale;
  t.quant.scale = scale_slot;
  t.quant.count = 1;
  t.quant.bit_width = 8;
  return t;
}

lsc_tensor f32_dev(const char* name, std::initializer_list<int64_t> shape, void* data) {
  lsc_tensor t{};
  t.name = name;
  t.ndim = 0;
  uint64_t n = 1;
  for (auto d : shape) {
    t.shape[t.ndim++] = d;
    n *= static_cast<uint64_t>(d);
  }
  t.dtype = LSC_DTYPE_F32;
  t.layout = LSC_LAYOUT_NCHW;
  t.location = LSC_MEM_DEVICE;
  t.data = data;
  t.nbytes = n * 4;
  return t;
}

// The filter of a stride-2 convolution re-expressed over the space-to-depth input: tap
// (r, s) = (2a + dy, 2b + dx) of the k x k filter moves to tap (a, b), channel (dy*2 + dx)*C + c
// of a ceil(k/2) x ceil(k/2) filter; taps past k are zero.
std::vector<float> s2d_filter(const std::vector<float>& w, int64_t co, int64_t c, int64_t k) {
  const int64_t kk = (k + 1) / 2;
  std::vector<float> w2(static_cast<size_t>(co * 4 * c * kk * kk), 0.0f);
  for (int64_t o = 0; o < co; ++o)
    for (int64_t dy = 0; dy < 2; ++dy)
      for (int64_t dx = 0; dx < 2; ++dx)
        for (int64_t a = 0; a < kk; ++a)
          for (int64_t b = 0; b < kk; ++b) {
            const int64_t r = 2 * a + dy, s = 2 * b + dx;
            if (r >= k || s >= k) continue;
            for (int64_t ci = 0; ci < c; ++ci)
              w2[static_cast<size_t>(((o * 4 * c + (dy * 2 + dx) * c + ci) * kk + a) * kk + b)] =
                  w[static_cast<size_t>(((o * c + ci) * k + r) * k + s)];
          }
  return w2;
}

// Lowers the fused graph to INT8 steps (shapes only; operators are compiled at calibration).
lsc_status lower_int8(QSession& q, const lsc_model& m) {
  if (m.inputs.size() != 1 || m.outputs.size() != 1)
    return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "INT8 session: one graph input and one output expected");
  const GraphIO& gi = m.inputs[0];
  if (gi.dtype != LSC_DTYPE_F32 || gi.shape.size() != 4)
    return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "INT8 session: the input must be f32 NCHW");
  for (auto d : gi.shape)
    if (d <= 0) return set_error(LSC_ERROR_SHAPE_MISMATCH, "INT8 session: the input needs static dimensions");
  q.in_shape = gi.shape;
  const int64_t N = gi.shape[0];
  std::map<std::string, int> alias;  // view tensor -> value id
  auto find = [&](const std::string& t) -> int {
    auto a = alias.find(t);
    if (a != alias.end()) return a->second;
    auto it = q.val_of.find(t);
    return it == q.val_of.end() ? -1 : it->second;
  };
  auto add_val = [&](const std::string& name, int64_t h, int64_t w, int64_t c) -> int {
    QVal v;
    v.name = name;
    v.n = N;
    v.h = h;
    v.w = w;
    v.c = c;
    v.w_store = w;
    v.c_store = c;  // layer outputs are stored as computed; the quantized input is padded below
    q.vals.push_back(v);
    const int id = static_cast<int>(q.vals.size()) - 1;
    q.val_of[name] = id;
    return id;
  };
  // how many nodes read a tensor
  auto readers = [&](const std::string& t) {
    int c = 0;
    for (const auto& n : m.nodes)
      for (const auto& x : n.in)
        if (x == t) ++c;
    for (const auto& o : m.outputs)
      if (o.name == t) ++c;
    return c;
  };
  std::set<size_t> absorbed;  // Add nodes fused into a convolution
  bool input_quantized = false;
  bool have_fc = false;
  for (size_t k = 0; k < m.nodes.size(); ++k) {
    if (absorbed.count(k)) continue;
    const Node& n = m.nodes[k];
    const lsc_op_desc& d = m.descs[k];
    if (have_fc) return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "INT8 session: node '%s' after the classifier", n.name.c_str());
    if (d.op_type == -1) {  // Flatten / Reshape of a pooled [N, C(,1,1)] tensor
      const int src = find(n.in[0]);
      if (src < 0) return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "INT8 session: view '%s' of an unknown tensor", n.name.c_str());
      if (!q.vals[src].flat)
        return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "INT8 session: only pooled tensors can be reshaped ('%s')", n.name.c_str());
      alias[n.out[0]] = src;
      continue;
    }
    QStep st;
    st.node = static_cast<int>(k);
    if (d.op_type == LSC_OP_CONV2D) {
      if (d.groups != 1 && d.groups != 0)
        return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "INT8 session: grouped Conv '%s'", n.name.c_str());
      const OnnxTensor& wt = m.inits.at(n.in[1]);
      const int64_t co = wt.dims[0], ci = wt.dims[1], kh = wt.dims[2], kw = wt.dims[3];
      int in = -1;
      if (n.in[0] == gi.name) {
        if (input_quantized) return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "INT8 session: the input feeds two nodes");
        input_quantized = true;
        QStep qs;
        qs.kind = QStep::kInput;
        const int64_t H = gi.shape[2], W = gi.shape[3], C = gi.shape[1];
        const int64_t p = d.pad_h;
        const bool s2d = d.stride_h == 2 && d.stride_w == 2 && kh == kw && d.pad_w == p && C <= 4 &&
                         d.dilation_h == 1 && d.dilation_w == 1 && (H + 2 * p) % 2 == 0 && (W + 2 * p) % 2 == 0 &&
                         d.pad_h_end_delta == 0 && d.pad_w_end_delta == 0 &&
                         (H + 2 * p - kh) / 2 + 1 == (H + 2 * p) / 2 - (kh + 1) / 2 + 1 &&
                         (W + 2 * p - kw) / 2 + 1 == (W + 2 * p) / 2 - (kw + 1) / 2 + 1;
        if (s2d) {
          const int64_t hs = (H + 2 * p) / 2, ws = (W + 2 * p) / 2;
          const int x = add_val(gi.name + ":q", hs, ws, 4 * C);
          q.vals[x].w_store = round_up(ws, 4);
          q.vals[x].c_store = 16;
          qs.s2d = st.s2d = true;
          qs.s2d_pad = st.s2d_pad = p;
          qs.s2d_extra = st.s2d_extra = q.vals[x].w_store - ws;
          qs.out = x;
        } else {
          qs.out = add_val(gi.name + ":q", H, W, C);
          q.vals[qs.out].c_store = round_up(C, 16);
        }
        q.steps.push_back(qs);
        in = qs.out;
      } else {
        in = find(n.in[0]);
        if (in < 0) return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "INT8 session: Conv '%s' reads an unknown tensor", n.name.c_str());
      }
      const QVal& x = q.vals[in];
      if (!st.s2d && x.c != ci)
        return set_error(LSC_ERROR_SHAPE_MISMATCH, "INT8 session: Conv '%s' expects %lld channels", n.name.c_str(), (long long)ci);
      if (x.flat || x.c_store % 16 != 0)
        return set_error(LSC_ERROR_UNSUPPORTED_LAYOUT,
                         "INT8 session: Conv '%s' reads %lld channels; int8 activations need a multiple of 16",
                         n.name.c_str(), (long long)x.c_store);
      int64_t oh, ow;
      if (st.s2d) {
        oh = x.h - (kh + 1) / 2 + 1;
        ow = x.w - (kw + 1) / 2 + 1;
      } else {
        oh = (x.h + 2 * d.pad_h + d.pad_h_end_delta - d.dilation_h * (kh - 1) - 1) / d.stride_h + 1;
        ow = (x.w + 2 * d.pad_w + d.pad_w_end_delta - d.dilation_w * (kw - 1) - 1) / d.stride_w + 1;
      }
      st.kind = QStep::kConv;
      st.in = in;
      st.act = d.activation;
      std::string out_name = n.out[0];
      // a following Add (+ ReLU) that only this convolution feeds becomes its residual
      if (readers(n.out[0]) == 1 && d.activation == LSC_ACT_NONE) {
        for (size_t j = k + 1; j < m.nodes.size(); ++j) {
          const Node& a = m.nodes[j];
          if (m.descs[j].op_type != LSC_OP_ADD) {
            bool reads = false;
            for (const auto& t : a.in) reads |= t == n.out[0];
            if (reads) break;
            continue;
          }
          if (a.in.size() != 2 || (a.in[0] != n.out[0] && a.in[1] != n.out[0])) continue;
          const std::string& other = a.in[0] == n.out[0] ? a.in[1] : a.in[0];
          const int r = find(other);
          if (r < 0 || q.vals[r].flat || q.vals[r].h != oh || q.vals[r].w != ow || q.vals[r].c != co) break;
          st.res = r;
          // Add + Relu arrives as FusionType::AddReLU (or an explicit activation)
          st.act = m.descs[j].fusion == LSC_FUSION_ADD_RELU ? LSC_ACT_RELU : m.descs[j].activation;
          out_name = a.out[0];
          absorbed.insert(j);
          break;
        }
      }
      st.out = add_val(out_name, oh, ow, co);
      q.steps.push_back(st);
      continue;
    }
    if (d.op_type == LSC_OP_MAXPOOL2D) {
      const int in = find(n.in[0]);
      if (in < 0 || q.vals[in].flat) return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "INT8 session: MaxPool '%s' input", n.name.c_str());
      const QVal& x = q.vals[in];
      st.kind = QStep::kMaxPool;
      st.in = in;
      if (d.kernel_h == d.kernel_w && d.stride_h == d.stride_w && d.pad_h == d.pad_w) {
        st.pool_k = d.kernel_h;
        st.pool_s = d.stride_h;
        st.pool_p = d.pad_h;
      }
      st.out = add_val(n.out[0], (x.h + 2 * d.pad_h - d.kernel_h) / d.stride_h + 1,
                       (x.w + 2 * d.pad_w - d.kernel_w) / d.stride_w + 1, x.c);
      q.steps.push_back(st);
      continue;
    }
    if (d.op_type == LSC_OP_GLOBAL_AVGPOOL2D) {
      const int in = find(n.in[0]);
      if (in < 0 || q.vals[in].flat) return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "INT8 session: GlobalAveragePool '%s' input", n.name.c_str());
      st.kind = QStep::kAvgPool;
      st.in = in;
      st.out = add_val(n.out[0], 1, 1, q.vals[in].c);
      q.vals[st.out].flat = true;
      q.steps.push_back(st);
      continue;
    }
    if (d.op_type == LSC_OP_FULLY_CONNECTED) {
      const int in = find(n.in[0]);
      if (in < 0 || !q.vals[in].flat) return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "INT8 session: FullyConnected '%s' needs a pooled input", n.name.c_str());
      if (n.out[0] != m.outputs[0].name)
        return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "INT8 session: the classifier '%s' must produce the graph output", n.name.c_str());
      st.kind = QStep::kFc;
      st.in = in;
      have_fc = true;
      q.steps.push_back(st);
      continue;
    }
    return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "INT8 session: operator %s ('%s') has no INT8 lowering",
                     n.op.c_str(), n.name.c_str());
  }
  if (!have_fc) return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "INT8 session: the graph must end in a Gemm / MatMul classifier");
  return LSC_SUCCESS;
}

// Schedule positions, second-stream steps and each value's live range.
// Step i is a ReLU convolution whose output only the 3x3 / 2 max pool (padding 1) of step i + 1
// reads, both on the main stream: they can run as one launch (lsc::execute_conv_pool decides
// whether the compiled convolution qualifies).
bool pool_fusable(const QSession& q, size_t i) {
  if (i + 1 >= q.steps.size()) return false;
  const QStep& c = q.steps[i];
  const QStep& m = q.steps[i + 1];
  if (c.kind != QStep::kConv || m.kind != QStep::kMaxPool || c.side || m.side || c.res >= 0 || m.in != c.out ||
      c.act != LSC_ACT_RELU || m.pool_k != 3 || m.pool_s != 2 || m.pool_p != 1)
    return false;
  for (size_t j = 0; j < q.steps.size(); ++j)
    if (j != i + 1 && (q.steps[j].in == c.out || q.steps[j].res == c.out)) return false;
  return true;
}

// The graph starts with the ResNet stem: the input quantized to space-to-depth (padding 3), read
// only by a ReLU convolution over 3 channels that yields 112 x 112 x 64 and whose output only a
// fused-able 3x3 / 2 max pool reads.  Such a stem can run as one launch from the f32 input
// (lsc::launch_stem_conv_pool_i8; prepare_stem checks the compiled parameters).
bool stem_shape_fusable(const QSession& q) {
  if (q.steps.size() < 3 || q.in_shape.size() != 4) return false;
  const QStep& in = q.steps[0];
  const QStep& cv = q.steps[1];
  if (in.kind != QStep::kInput || !in.s2d || in.s2d_pad != 3 || cv.kind != QStep::kConv || !cv.s2d ||
      cv.in != in.out || !pool_fusable(q, 1))
    return false;
  if (q.in_shape[1] != 3 || q.in_shape[2] != 224 || q.in_shape[3] != 224) return false;
  const QVal& co = q.vals[cv.out];
  const QVal& po = q.vals[q.steps[2].out];
  if (co.h != 112 || co.w != 112 || co.c != 64 || co.c_store != 64 || co.w_store != 112 || po.h != 56 ||
      po.w != 56 || po.c_store != 64 || po.w_store != 56 || po.flat)
    return false;
  for (size_t j = 2; j < q.steps.size(); ++j)
    if (q.steps[j].in == in.out || q.steps[j].res == in.out) return false;
  return true;
}

void schedule_int8(QSession& q) {
  int pos = 0;
  int prev_conv_in = -1;
  for (size_t i = 0; i < q.steps.size(); ++i) {
    QStep& s = q.steps[i];
    s.side = false;
    // a convolution reading the same tensor as the convolution just before it runs beside it
    if (q.concurrent && s.kind == QStep::kConv && i > 0 && q.steps[i - 1].kind == QStep::kConv &&
        !q.steps[i - 1].side && s.in == prev_conv_in && s.res < 0) {
      s.side = true;
      s.pos = q.steps[i - 1].pos;
    } else {
      s.pos = ++pos;
    }
    prev_conv_in = s.kind == QStep::kConv ? s.in : -1;
  }
  for (auto& v : q.vals) v.def = v.last = -1;
  for (auto& s : q.steps) {
    if (s.out >= 0) q.vals[s.out].def = s.pos;
    for (int r : {s.in, s.res})
      if (r >= 0) q.vals[r].last = std::max(q.vals[r].last, s.pos);
  }
  // a max pool fused into the convolution before it is written while that convolution still
  // reads its input: its output lives from the convolution on
  for (size_t i = 0; i + 1 < q.steps.size(); ++i)
    if (pool_fusable(q, i)) q.vals[q.steps[i + 1].out].def = q.steps[i].pos;
  // ... and a stem run as one launch writes it while the input is being quantized
  if (stem_shape_fusable(q)) q.vals[q.steps[2].out].def = q.steps[0].pos;
  for (auto& v : q.vals)
    if (v.last < v.def) v.last = v.def;
}

// Offsets in one block: largest first, lowest offset clear of every placed value whose live
// range overlaps.
uint64_t plan_offsets(QSession& q) {
  std::vector<int> order(q.vals.size());
  for (size_t i = 0; i < order.size(); ++i) order[i] = static_cast<int>(i);
  std::sort(order.begin(), order.end(), [&](int a, int b) { return q.vals[a].bytes() > q.vals[b].bytes(); });
  std::vector<int> placed;
  uint64_t total = 0;
  for (int id : order) {
    QVal& v = q.vals[id];
    const int64_t size = round_up(v.bytes(), 256);
    std::vector<std::pair<int64_t, int64_t>> busy;
    for (int p : placed) {
      const QVal& u = q.vals[p];
      if (u.def <= v.last && v.def <= u.last) busy.emplace_back(u.offset, u.offset + round_up(u.bytes(), 256));
    }
    std::sort(busy.begin(), busy.end());
    int64_t off = 0;
    for (const auto& b : busy) {
      if (off + size <= b.first) break;
      off = std::max(off, b.second);
    }
    v.offset = off;
    placed.push_back(id);
    total = std::max<uint64_t>(total, static_cast<uint64_t>(off + size));
  }
  return total;
}

// find_scale_zp (symmetric, QInt8) of a device f32 array, read back to the host.
lsc_status calibrate_scale(lsc_backend* be, const float* x, int64_t n, cudaStream_t st, float* scale) {
  lsc_memory_block b{};
  lsc_status s = lsc_allocate(be, 64, 256, &b);
  if (s) return s;
  char* base = static_cast<char*>(b.ptr);
  s = lsc::launch_find_scale_zp(x, n, LSC_DTYPE_QINT8, 1, base, 16, reinterpret_cast<float*>(base + 16),
                                reinterpret_cast<int32_t*>(base + 32), st);
  if (!s) {
    cudaError_t e = cudaMemcpyAsync(scale, base + 16, 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) s = lsc::cuda_error(e, "calibration scale");
  }
  lsc_deallocate(be, &b);
  return s;
}

// Compiles every step with the calibrated scales, running the calibration batch through
// the network layer by layer (`x` device f32 NCHW of the input shape).
lsc_status calibrate_int8(QSession& q, const lsc_model& m, const float* x, cudaStream_t st) {
  lsc_backend* be = q.be;
  const int64_t in_count = count_of(q.in_shape);
  lsc_status s = calibrate_scale(be, x, in_count, st, &q.in_scale);
  if (s) return s;
  int64_t scratch_elems = 0;
  for (const auto& v : q.vals) scratch_elems = std::max(scratch_elems, v.n * v.h * v.w * v.c_store);
  scratch_elems = std::max(scratch_elems, q.in_shape[0] * 4096);
  lsc_memory_block sb{};
  if ((s = lsc_allocate(be, static_cast<uint64_t>(scratch_elems) * 4, 256, &sb))) return s;
  float* scratch = static_cast<float*>(sb.ptr);
  auto fail = [&](lsc_status e) {
    lsc_deallocate(be, &sb);
    return e;
  };
  float sc_a = 0.0f, sc_b = 0.0f, sc_c = 0.0f;
  for (auto& stp : q.steps) {
    const Node* n = stp.node >= 0 ? &m.nodes[stp.node] : nullptr;
    if (stp.kind == QStep::kInput) {
      QVal& o = q.vals[stp.out];
      o.scale = q.in_scale;
      lsc_op_desc d = base_desc(LSC_OP_QUANTIZE);
      d.rounding = q.rounding;
      if (stp.s2d) {
        d.stride_h = d.stride_w = 2;
        d.pad_h = d.pad_w = static_cast<int32_t>(stp.s2d_pad);
        d.pad_w_end_delta = static_cast<int32_t>(2 * stp.s2d_extra);
      }
      lsc_tensor xi = f32_dev("input", {q.in_shape[0], q.in_shape[1], q.in_shape[2], q.in_shape[3]},
                              const_cast<float*>(x));
      lsc_tensor xo = q_tensor(o, q.ptr(stp.out), &sc_a);
      if ((s = lsc_compile_operator(be, &d, &xi, 1, &xo, 1, &stp.op))) return fail(s);
      if ((s = lsc_execute(be, stp.op, &xi, 1, &xo, 1, st))) return fail(s);
      continue;
    }
    if (stp.kind == QStep::kConv) {
      const QVal& xv = q.vals[stp.in];
      QVal& ov = q.vals[stp.out];
      const OnnxTensor& wt = m.inits.at(n->in[1]);
      const int64_t co = wt.dims[0], ci = wt.dims[1], kh = wt.dims[2];
      lsc_op_desc d = m.descs[stp.node];
      d.activation = stp.act;
      d.rounding = q.rounding;
      d.output_dtype = LSC_DTYPE_QINT8;
      d.output_scale = 1.0f;
      std::vector<float> w2;
      std::vector<int64_t> wshape = wt.dims;
      const float* wdata = wt.f.data();
      if (stp.s2d) {
        w2 = s2d_filter(wt.f, co, ci, kh);
        const int64_t kk = (kh + 1) / 2;
        wshape = {co, 4 * ci, kk, kk};
        wdata = w2.data();
        d.stride_h = d.stride_w = 1;
        d.pad_h = d.pad_w = 0;
        d.pad_h_end_delta = 0;
        d.pad_w_end_delta = -static_cast<int32_t>(stp.s2d_extra);
      }
      std::vector<lsc_tensor> cin;
      cin.push_back(q_tensor(xv, q.ptr(stp.in), &sc_a));
      cin.push_back(host_f32(n->in[1].c_str(), wshape, wdata));
      std::vector<float> zero_bias;
      if (n->in.size() > 2 && !n->in[2].empty()) {
        const OnnxTensor& bt = m.inits.at(n->in[2]);
        cin.push_back(host_f32(n->in[2].c_str(), bt.dims, bt.f.data()));
      } else {
        zero_bias.assign(static_cast<size_t>(co), 0.0f);
        cin.push_back(host_f32("bias", {co}, zero_bias.data()));
      }
      for (const auto& b : n->bn) {
        const OnnxTensor& t = m.inits.at(b);
        cin.push_back(host_f32(b.c_str(), t.dims, t.f.data()));
      }
      lsc_tensor yo = q_tensor(ov, q.ptr(stp.out), &sc_b);
      if ((s = lsc_compile_operator(be, &d, cin.data(), static_cast<int32_t>(cin.size()), &yo, 1, &stp.op)))
        return fail(s);
      std::vector<lsc_tensor> ein{q_tensor(xv, q.ptr(stp.in), &sc_a)};
      if (stp.res >= 0) ein.push_back(q_tensor(q.vals[stp.res], q.ptr(stp.res), &sc_c));
      lsc_tensor yf = f32_dev(ov.name.c_str(), {ov.n, ov.h, ov.w, ov.c_store}, scratch);
      yf.layout = LSC_LAYOUT_NHWC;
      if ((s = lsc_execute(be, stp.op, ein.data(), static_cast<int32_t>(ein.size()), &yf, 1, st))) return fail(s);
      if ((s = calibrate_scale(be, scratch, ov.n * ov.h * ov.w * ov.c_store, st, &ov.scale))) return fail(s);
      yo = q_tensor(ov, q.ptr(stp.out), &sc_b);
      if ((s = lsc_execute(be, stp.op, ein.data(), static_cast<int32_t>(ein.size()), &yo, 1, st))) return fail(s);
      continue;
    }
    if (stp.kind == QStep::kMaxPool) {
      const QVal& xv = q.vals[stp.in];
      QVal& ov = q.vals[stp.out];
      ov.scale = xv.scale;
      lsc_op_desc d = m.descs[stp.node];
      lsc_tensor xi = q_tensor(xv, q.ptr(stp.in), &sc_a);
      lsc_tensor xo = q_tensor(ov, q.ptr(stp.out), &sc_b);
      if ((s = lsc_compile_operator(be, &d, &xi, 1, &xo, 1, &stp.op))) return fail(s);
      if ((s = lsc_execute(be, stp.op, &xi, 1, &xo, 1, st))) return fail(s);
      continue;
    }
    if (stp.kind == QStep::kAvgPool) {
      const QVal& xv = q.vals[stp.in];
      QVal& ov = q.vals[stp.out];
      lsc_op_desc d = m.descs[stp.node];
      d.rounding = q.rounding;
      d.output_scale = 1.0f;
      lsc_tensor xi = q_tensor(xv, q.ptr(stp.in), &sc_a);
      lsc_tensor yf = f32_dev(ov.name.c_str(), {ov.n, ov.c_store}, scratch);
      if ((s = lsc_compile_operator(be, &d, &xi, 1, &yf, 1, &stp.op))) return fail(s);
      if ((s = lsc_execute(be, stp.op, &xi, 1, &yf, 1, st))) return fail(s);
      if ((s = calibrate_scale(be, scratch, ov.n * ov.c_store, st, &ov.scale))) return fail(s);
      lsc_tensor yo = q_tensor(ov, q.ptr(stp.out), &sc_b);
      if ((s = lsc_execute(be, stp.op, &xi, 1, &yo, 1, st))) return fail(s);
      continue;
    }
    // kFc: INT8 FullyConnected, f32 logits (Gemm transB = 1 keeps W as [N, K])
    const QVal& xv = q.vals[stp.in];
    const OnnxTensor& wt = m.inits.at(n->in[1]);
    const bool trans_b = n->op == "Gemm" && n->attr_i("transB", 0) != 0;
    const int64_t kdim = trans_b ? wt.dims[1] : wt.dims[0], ndim = trans_b ? wt.dims[0] : wt.dims[1];
    if (kdim != xv.c) return fail(set_error(LSC_ERROR_SHAPE_MISMATCH, "INT8 session: classifier K mismatch"));
    std::vector<float> wnk;
    const float* wdata = wt.f.data();
    if (!trans_b) {
      wnk.resize(static_cast<size_t>(kdim * ndim));
      for (int64_t a = 0; a < kdim; ++a)
        for (int64_t b = 0; b < ndim; ++b) wnk[static_cast<size_t>(b * kdim + a)] = wt.f[static_cast<size_t>(a * ndim + b)];
      wdata = wnk.data();
    }
    std::vector<float> zero_bias(static_cast<size_t>(ndim), 0.0f);
    const float* bdata = zero_bias.data();
    if (n->in.size() > 2 && !n->in[2].empty()) bdata = m.inits.at(n->in[2]).f.data();
    lsc_op_desc d = base_desc(LSC_OP_FULLY_CONNECTED);
    d.rounding = q.rounding;
    QVal xin = xv;
    xin.c_store = xv.c;  // the FC reads [N, K]: K = the pooled channels (multiple of 16 here)
    if (xv.c_store != xv.c) return fail(set_error(LSC_ERROR_UNSUPPORTED_LAYOUT, "INT8 session: classifier input channels must be a multiple of 16"));
    lsc_tensor cin[3] = {q_tensor(xin, q.ptr(stp.in), &sc_a), host_f32("fc.w", {ndim, kdim}, wdata),
                         host_f32("fc.b", {ndim}, bdata)};
    lsc_tensor yo = f32_dev("logits", {xv.n, ndim}, q.out_buf);
    if ((s = lsc_compile_operator(be, &d, cin, 3, &yo, 1, &stp.op))) return fail(s);
    if ((s = lsc_execute(be, stp.op, cin, 1, &yo, 1, st))) return fail(s);
    q.out_classes = ndim;
  }
  lsc_deallocate(be, &sb);
  cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return lsc::cuda_error(e, "INT8 session calibration");
  return LSC_SUCCESS;
}

// Launches every step on `main` (and the side stream) reading the input from `in`.  A side
// step forks from `main` before the step it runs beside, so both start from the same point,
// and the next step joins it.
lsc_status enqueue_int8(QSession& q, const float* in, cudaStream_t main) {
  float sc_a = 0.0f, sc_b = 0.0f, sc_c = 0.0f;
  bool pool_done = false;
  int stem_left = 0;  // steps the fused stem launch has done
  size_t fork_i = 0, join_i = 0;
  bool side_open = false;
  for (size_t i = 0; i < q.steps.size(); ++i) {
    QStep& stp = q.steps[i];
    lsc_status s;
    if (side_open && !stp.side) {
      LSC_CUDA_TRY(cudaEventRecord(q.join_ev[join_i], q.side_stream));
      LSC_CUDA_TRY(cudaStreamWaitEvent(main, q.join_ev[join_i], 0));
      ++join_i;
      side_open = false;
    }
    if (i + 1 < q.steps.size() && q.steps[i + 1].side) {
      LSC_CUDA_TRY(cudaEventRecord(q.fork_ev[fork_i], main));
      LSC_CUDA_TRY(cudaStreamWaitEvent(q.side_stream, q.fork_ev[fork_i], 0));
      ++fork_i;
    }
    cudaStream_t st = stp.side ? q.side_stream : main;
    side_open |= stp.side;
    if (pool_done) {
      pool_done = false;
      continue;
    }
    if (stem_left > 0) {
      --stem_left;
      continue;
    }
    if (stp.kind == QStep::kInput && q.stem_fused && i == 0) {
      // input quantize, stem convolution and max pool in one launch: the space-to-depth input
      // and the convolution output are not written
      const QStep& cv = q.steps[1];
      const QStep& pool = q.steps[2];
      s = lsc::launch_stem_conv_pool_i8(in, q.in_shape[0], static_cast<const int8_t*>(q.stem_w), cv.op->bias_i32,
                                        cv.op->scale, q.vals[stp.out].scale, stp.op->rounding,
                                        q.vals[cv.out].scale, cv.op->rounding, static_cast<int8_t*>(q.ptr(pool.out)), st);
      if (s) return s;
      stem_left = 2;
      continue;
    }
    if (stp.kind == QStep::kInput) {
      lsc_tensor xi = f32_dev("input", {q.in_shape[0], q.in_shape[1], q.in_shape[2], q.in_shape[3]}, const_cast<float*>(in));
      lsc_tensor xo = q_tensor(q.vals[stp.out], q.ptr(stp.out), &sc_b);
      if ((s = lsc_execute(q.be, stp.op, &xi, 1, &xo, 1, st))) return s;
      continue;
    }
    lsc_tensor xi = q_tensor(q.vals[stp.in], q.ptr(stp.in), &sc_a);
    if (stp.kind == QStep::kFc) {
      lsc_tensor yo = f32_dev("logits", {q.vals[stp.in].n, q.out_classes}, q.out_buf);
      if ((s = lsc_execute(q.be, stp.op, &xi, 1, &yo, 1, st))) return s;
      continue;
    }
    lsc_tensor yo = q_tensor(q.vals[stp.out], q.ptr(stp.out), &sc_b);
    if (pool_fusable(q, i)) {
      // the stem's convolution and the 3x3 / 2 max pool after it in one launch; the conv
      // output (only the pool reads it) is not written
      const QStep& pool = q.steps[i + 1];
      lsc_tensor po = q_tensor(q.vals[pool.out], q.ptr(pool.out), &sc_c);
      s = lsc::execute_conv_pool(stp.op, xi, po, st);
      if (s == LSC_SUCCESS) {
        pool_done = true;  // the next step (the pool) has run
        continue;
      }
      if (s != LSC_ERROR_UNSUPPORTED_OPERATOR) return s;
    }
    if (stp.kind == QStep::kConv && stp.res >= 0) {
      lsc_tensor ins[2] = {xi, q_tensor(q.vals[stp.res], q.ptr(stp.res), &sc_c)};
      if ((s = lsc_execute(q.be, stp.op, ins, 2, &yo, 1, st))) return s;
    } else {
      if ((s = lsc_execute(q.be, stp.op, &xi, 1, &yo, 1, st))) return s;
    }
  }
  if (side_open) {
    LSC_CUDA_TRY(cudaEventRecord(q.join_ev[join_i], q.side_stream));
    LSC_CUDA_TRY(cudaStreamWaitEvent(main, q.join_ev[join_i], 0));
  }
  return LSC_SUCCESS;
}

// Decides whether the stem runs as one launch and builds that kernel's filter image from the
// compiled space-to-depth convolution.  Besides the shapes (stem_shape_fusable), the fused form
// pools the int32 accumulators before requantizing, which equals pooling the int8 codes when
// every channel scale is positive and acc + bias cannot wrap (|acc| < 2^22 for 147 int8 taps);
// otherwise, or with LSC_FUSED_STEM=0 in the environment, the stem keeps its separate launches.
lsc_status prepare_stem(QSession& q) {
  q.stem_fused = false;
  const char* env = getenv("LSC_FUSED_STEM");
  if ((env && env[0] == '0') || !stem_shape_fusable(q)) return LSC_SUCCESS;
  const lsc_op* op = q.steps[1].op;
  lsc::DeviceState* ds = lsc::current_device_state();
  if (!op || !ds || ds->cc_major != 10 || op->kind != OpKind::kConvI8 || op->act != LSC_ACT_RELU || op->n != 64 ||
      op->kh != 4 || op->kw != 4 || op->kp != 16 || !op->w || !op->scale)
    return LSC_SUCCESS;
  if (!(q.vals[q.steps[1].out].scale > 0.0f)) return LSC_SUCCESS;
  std::vector<float> scale(64);
  std::vector<int32_t> bias(64, 0);
  std::vector<int8_t> w(64 * 4 * 4 * 16), img(static_cast<size_t>(lsc::kStemFilterBytes));
  LSC_CUDA_TRY(cudaMemcpy(scale.data(), op->scale, 64 * 4, cudaMemcpyDeviceToHost));
  if (op->bias_i32) LSC_CUDA_TRY(cudaMemcpy(bias.data(), op->bias_i32, 64 * 4, cudaMemcpyDeviceToHost));
  LSC_CUDA_TRY(cudaMemcpy(w.data(), op->w, w.size(), cudaMemcpyDeviceToHost));
  for (int c = 0; c < 64; ++c)
    if (!(scale[static_cast<size_t>(c)] > 0.0f) || !std::isfinite(scale[static_cast<size_t>(c)]) ||
        bias[static_cast<size_t>(c)] > (1 << 30) || bias[static_cast<size_t>(c)] < -(1 << 30))
      return LSC_SUCCESS;
  lsc::stem_filter_image(w.data(), img.data());
  if (!(q.stem_w = q.be->arena.alloc(static_cast<size_t>(lsc::kStemFilterBytes), 256)))
    return set_error(LSC_ERROR_OUT_OF_MEMORY, "INT8 session: no arena room for the stem filter");
  LSC_CUDA_TRY(cudaMemcpy(q.stem_w, img.data(), img.size(), cudaMemcpyHostToDevice));
  q.stem_fused = true;
  return LSC_SUCCESS;
}

lsc_status capture_int8(QSession& q) {
  size_t sides = 0;
  for (const auto& s : q.steps) sides += s.side ? 1 : 0;
  q.fork_ev.resize(sides);
  q.join_ev.resize(sides + 1);
  for (auto& e : q.fork_ev) LSC_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  for (auto& e : q.join_ev) LSC_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  for (int k = 0; k < 2; ++k) {
    LSC_CUDA_TRY(cudaStreamBeginCapture(q.cap_stream, cudaStreamCaptureModeThreadLocal));
    lsc_status s = enqueue_int8(q, static_cast<const float*>(q.in_slot[k]), q.cap_stream);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(q.cap_stream, &g);
    if (s) {
      if (g) cudaGraphDestroy(g);
      return s;
    }
    if (e != cudaSuccess) return lsc::cuda_error(e, "INT8 session graph capture");
    e = cudaGraphInstantiate(&q.exec[k], g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return lsc::cuda_error(e, "INT8 session graph instantiation");
  }
  return LSC_SUCCESS;
}

lsc_status build_int8(QSession& q, const lsc_model& m, const lsc_tensor* calib) {
  lsc_status s = lower_int8(q, m);
  if (s) return s;
  schedule_int8(q);
  uint64_t separate = 0;
  for (const auto& v : q.vals) separate += static_cast<uint64_t>(round_up(v.bytes(), 256));
  q.unplanned_bytes = separate;
  if (q.plan_memory) {
    q.planned_bytes = plan_offsets(q);
    q.act_block = q.be->arena.alloc(q.planned_bytes, 256);
    if (!q.act_block) return set_error(LSC_ERROR_OUT_OF_MEMORY, "INT8 session: no arena room for %llu activation bytes",
                                       (unsigned long long)q.planned_bytes);
  } else {
    q.planned_bytes = separate;
    for (const auto& v : q.vals) {
      void* p = q.be->arena.alloc(static_cast<size_t>(round_up(v.bytes(), 256)), 256);
      if (!p) return set_error(LSC_ERROR_OUT_OF_MEMORY, "INT8 session: no arena room for '%s'", v.name.c_str());
      q.act_blocks.push_back(p);
    }
  }
  const uint64_t in_bytes = static_cast<uint64_t>(count_of(q.in_shape)) * 4;
  for (int k = 0; k < 2; ++k)
    if (!(q.in_slot[k] = q.be->arena.alloc(in_bytes, 256)))
      return set_error(LSC_ERROR_OUT_OF_MEMORY, "INT8 session: no arena room for the input");
  // the classifier's width is known once it is compiled; room for up to 64 Ki classes
  const uint64_t out_bytes = static_cast<uint64_t>(q.in_shape[0]) * 65536 * 4;
  const Node& fc = m.nodes[q.steps.back().node];
  const OnnxTensor& fw = m.inits.at(fc.in[1]);
  const bool trans_b = fc.op == "Gemm" && fc.attr_i("transB", 0) != 0;
  const int64_t classes = trans_b ? fw.dims[0] : fw.dims[1];
  if (classes > 65536) return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "INT8 session: more than 65536 classes");
  (void)out_bytes;
  if (!(q.out_buf = q.be->arena.alloc(static_cast<size_t>(q.in_shape[0] * classes * 4), 256)))
    return set_error(LSC_ERROR_OUT_OF_MEMORY, "INT8 session: no arena room for the output");
  LSC_CUDA_TRY(cudaStreamCreateWithFlags(&q.cap_stream, cudaStreamNonBlocking));
  LSC_CUDA_TRY(cudaStreamCreateWithFlags(&q.side_stream, cudaStreamNonBlocking));
  LSC_CUDA_TRY(cudaStreamCreateWithFlags(&q.copy_stream, cudaStreamNonBlocking));
  for (int k = 0; k < 2; ++k) {
    LSC_CUDA_TRY(cudaEventCreateWithFlags(&q.slot_loaded[k], cudaEventDisableTiming));
    LSC_CUDA_TRY(cudaEventCreateWithFlags(&q.slot_free[k], cudaEventDisableTiming));
  }
  // the calibration batch, staged into input slot 0 (host or device f32 of the input's shape)
  const lsc_tensor& c = *calib;
  bool ok = c.dtype == LSC_DTYPE_F32 && c.ndim == 4 && c.data;
  for (int i = 0; ok && i < 4; ++i) ok = c.shape[i] == q.in_shape[static_cast<size_t>(i)];
  if (!ok) return set_error(LSC_ERROR_SHAPE_MISMATCH, "INT8 session: the calibration batch must be f32 of the input's shape");
  LSC_CUDA_TRY(cudaMemcpyAsync(q.in_slot[0], c.data, in_bytes,
                               c.location == LSC_MEM_DEVICE ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                               q.cap_stream));
  if ((s = calibrate_int8(q, m, static_cast<const float*>(q.in_slot[0]), q.cap_stream))) return s;
  if ((s = prepare_stem(q))) return s;
  return capture_int8(q);
}

// Copies the input into slot k on `st` (nothing when it already lives there).
lsc_status stage_input(QSession& q, const lsc_tensor& t, int k, cudaStream_t st) {
  const uint64_t bytes = static_cast<uint64_t>(count_of(q.in_shape)) * 4;
  bool ok = t.dtype == LSC_DTYPE_F32 && t.ndim == 4 && t.data && (!t.nbytes || t.nbytes >= bytes);
  for (int i = 0; ok && i < 4; ++i) ok = t.shape[i] == q.in_shape[static_cast<size_t>(i)];
  if (!ok) return set_error(LSC_ERROR_SHAPE_MISMATCH, "lsc_session_run: the input must be f32 of the model's input shape");
  if (t.data == q.in_slot[k]) return LSC_SUCCESS;
  LSC_CUDA_TRY(cudaMemcpyAsync(q.in_slot[k], t.data, bytes,
                               t.location == LSC_MEM_DEVICE ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, st));
  return LSC_SUCCESS;
}

lsc_status fetch_output(QSession& q, lsc_tensor& t, cudaStream_t st) {
  const uint64_t bytes = static_cast<uint64_t>(q.in_shape[0] * q.out_classes) * 4;
  if (!t.data || (t.nbytes && t.nbytes < bytes))
    return set_error(LSC_ERROR_SHAPE_MISMATCH, "lsc_session_run: the output needs %llu bytes", (unsigned long long)bytes);
  t.ndim = 2;
  t.shape[0] = q.in_shape[0];
  t.shape[1] = q.out_classes;
  t.dtype = LSC_DTYPE_F32;
  if (t.data == q.out_buf) return LSC_SUCCESS;
  LSC_CUDA_TRY(cudaMemcpyAsync(t.data, q.out_buf, bytes,
                               t.location == LSC_MEM_DEVICE ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, st));
  return LSC_SUCCESS;
}

}  // namespace

void destroy_qsession(QSession* q) { delete q; }

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
  if (s->q) {
    // INT8: input slot 0, the captured graph, the output; host buffers complete on return
    if (n_inputs != 1 || n_outputs != 1 || !inputs || !outputs)
      return set_error(LSC_ERROR_INVALID_ARGUMENT, "lsc_session_run: one input and one output");
    QSession& q = *s->q;
    lsc::DeviceGuard guard(s->be->device);
    if (!guard.ok()) return LSC_ERROR_DEVICE_ERROR;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    lsc_status r = stage_input(q, inputs[0], 0, st);
    if (r) return r;
    LSC_CUDA_TRY(cudaGraphLaunch(q.exec[0], st));
    if ((r = fetch_output(q, outputs[0], st))) return r;
    if (inputs[0].location == LSC_MEM_HOST || outputs[0].location == LSC_MEM_HOST)
      LSC_CUDA_TRY(cudaStreamSynchronize(st));
    return LSC_SUCCESS;
  }
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


lsc_status lsc_session_create_ex(lsc_backend* backend, const lsc_model* model, const lsc_session_options* options,
                                 lsc_session** out) {
  if (!options || options->precision == LSC_PRECISION_F32) return lsc_session_create(backend, model, out);
  if (!backend || !model || !out) return set_error(LSC_ERROR_INVALID_ARGUMENT, "lsc_session_create_ex: null argument");
  *out = nullptr;
  if (options->precision != LSC_PRECISION_INT8)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "lsc_session_create_ex: unknown precision %d", options->precision);
  if (!options->calibration)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "lsc_session_create_ex: an INT8 session needs a calibration batch");
  lsc::DeviceGuard guard(backend->device);
  if (!guard.ok()) return LSC_ERROR_DEVICE_ERROR;
  std::unique_ptr<lsc_session> s(new (std::nothrow) lsc_session());
  if (!s) return set_error(LSC_ERROR_OUT_OF_MEMORY, "lsc_session_create_ex: out of host memory");
  backend->retain();
  s->be = backend;
  s->model = model;
  s->q = new (std::nothrow) QSession();
  if (!s->q) return set_error(LSC_ERROR_OUT_OF_MEMORY, "lsc_session_create_ex: out of host memory");
  QSession& q = *s->q;
  q.be = backend;
  q.rounding = options->rounding >= 0 ? options->rounding : backend->cfg.rounding;
  q.concurrent = options->concurrent != 0;
  q.plan_memory = options->plan_memory != 0;
  lsc_status st = build_int8(q, *model, options->calibration);
  if (st) return st;
  *out = s.release();
  return LSC_SUCCESS;
}

lsc_status lsc_session_run_async(lsc_session* s, const lsc_tensor* inputs, uint32_t n_inputs, lsc_tensor* outputs,
                                 uint32_t n_outputs, lsc_stream stream) {
  if (!s) return set_error(LSC_ERROR_INVALID_ARGUMENT, "lsc_session_run_async: null session");
  if (!s->q) return set_error(LSC_ERROR_NOT_IMPLEMENTED, "lsc_session_run_async: INT8 sessions only");
  if (n_inputs != 1 || n_outputs != 1 || !inputs || !outputs)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "lsc_session_run_async: one input and one output");
  QSession& q = *s->q;
  lsc::DeviceGuard guard(s->be->device);
  if (!guard.ok()) return LSC_ERROR_DEVICE_ERROR;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int k = q.next_slot;
  q.next_slot ^= 1;
  lsc_status r;
  if (inputs[0].location == LSC_MEM_HOST) {
    // host data is ready now: upload on the copy stream once slot k's last reader has finished
    LSC_CUDA_TRY(cudaStreamWaitEvent(q.copy_stream, q.slot_free[k], 0));
    if ((r = stage_input(q, inputs[0], k, q.copy_stream))) return r;
    LSC_CUDA_TRY(cudaEventRecord(q.slot_loaded[k], q.copy_stream));
    LSC_CUDA_TRY(cudaStreamWaitEvent(st, q.slot_loaded[k], 0));
  } else if ((r = stage_input(q, inputs[0], k, st))) {
    return r;
  }
  LSC_CUDA_TRY(cudaGraphLaunch(q.exec[k], st));
  LSC_CUDA_TRY(cudaEventRecord(q.slot_free[k], st));
  return fetch_output(q, outputs[0], st);
}

lsc_status lsc_session_io_buffer(lsc_session* s, int32_t is_output, uint32_t index, void** device_ptr,
                                 uint64_t* bytes) {
  if (!s || !device_ptr || index != 0) return set_error(LSC_ERROR_INVALID_ARGUMENT, "lsc_session_io_buffer: bad arguments");
  if (!s->q) return set_error(LSC_ERROR_NOT_IMPLEMENTED, "lsc_session_io_buffer: INT8 sessions only");
  QSession& q = *s->q;
  *device_ptr = is_output ? q.out_buf : q.in_slot[0];
  if (bytes)
    *bytes = static_cast<uint64_t>(is_output ? q.in_shape[0] * q.out_classes : count_of(q.in_shape)) * 4;
  return LSC_SUCCESS;
}

lsc_status lsc_session_memory_plan(const lsc_session* s, uint64_t* planned_bytes, uint64_t* unplanned_bytes,
                                   uint32_t* values) {
  if (!s) return set_error(LSC_ERROR_INVALID_ARGUMENT, "lsc_session_memory_plan: null session");
  if (!s->q) return set_error(LSC_ERROR_NOT_IMPLEMENTED, "lsc_session_memory_plan: INT8 sessions only");
  if (planned_bytes) *planned_bytes = s->q->planned_bytes;
  if (unplanned_bytes) *unplanned_bytes = s->q->unplanned_bytes;
  if (values) *values = static_cast<uint32_t>(s->q->vals.size());
  return LSC_SUCCESS;
}

lsc_status lsc_session_value(const lsc_session* s, const char* tensor_name, float* scale, void** device_ptr,
                             lsc_tensor* desc) {
  if (!s || !tensor_name) return set_error(LSC_ERROR_INVALID_ARGUMENT, "lsc_session_value: null argument");
  if (!s->q) return set_error(LSC_ERROR_NOT_IMPLEMENTED, "lsc_session_value: INT8 sessions only");
  const QSession& q = *s->q;
  auto it = q.val_of.find(tensor_name);
  if (it == q.val_of.end())
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "lsc_session_value: no int8 tensor '%s'", tensor_name);
  const QVal& v = q.vals[it->second];
  if (scale) *scale = v.scale;
  if (device_ptr) *device_ptr = q.ptr(it->second);
  if (desc) {
    float dummy = 0.0f;
    *desc = q_tensor(v, q.ptr(it->second), &dummy);
    desc->name = nullptr;
    desc->quant = lsc_quant{};
  }
  return LSC_SUCCESS;
}

}  // extern "C"
