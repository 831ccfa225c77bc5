// CactusGraph on the B200: node construction follows the reference builders
// (cactus/graph/graph_builder.cpp: add_node :572-596, matmul :61-81, index :123-159, ...);
// execute() walks the nodes in insertion order (graph_execute.cpp:231-395) and dispatches
// each node to the C-ABI kernels of include/cactus_b200.h on the graph's stream
// (compute_matmul_node graph_ops_nn.cpp:129-231, compute_embedding_node
// graph_ops_tensor.cpp:226-331, compute_sample_node graph_ops_sample.cpp:8-39, ...).
#include <cuda_runtime.h>

#include <chrono>
#include <cmath>
#include <cstring>
#include <fstream>
#include <iomanip>
#include <random>
#include <sstream>

#include "../../../include/cactus/graph.h"
#include "../../../include/cactus_b200.h"
#include "../engine/weights_io.h"

namespace {
void ck(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}
void kck(int rc, const char* what) {
    if (rc != 0) throw std::runtime_error(std::string(what) + ": " + cactus_cuda_last_error());
}
bool is_device_ptr(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}
size_t prod(const std::vector<size_t>& s) {
    size_t n = 1;
    for (size_t v : s) n *= v;
    return s.empty() ? 0 : n;
}
const char* op_name(OpType t) {
    switch (t) {
        case OpType::INPUT: return "INPUT";
        case OpType::ADD: return "ADD";
        case OpType::ADD_CLIPPED: return "ADD_CLIPPED";
        case OpType::MULTIPLY: return "MULTIPLY";
        case OpType::MATMUL: return "MATMUL";
        case OpType::TRANSPOSE: return "TRANSPOSE";
        case OpType::RESHAPE: return "RESHAPE";
        case OpType::EMBEDDING: return "EMBEDDING";
        case OpType::RMS_NORM: return "RMS_NORM";
        case OpType::LAYERNORM: return "LAYERNORM";
        case OpType::CONV1D_CAUSAL: return "CONV1D_CAUSAL";
        case OpType::CONV1D_K3: return "CONV1D_K3";
        case OpType::ROPE: return "ROPE";
        case OpType::SOFTMAX: return "SOFTMAX";
        case OpType::ATTENTION: return "ATTENTION";
        case OpType::ATTENTION_INT8_HYBRID: return "ATTENTION_INT8_HYBRID";
        case OpType::SCALAR_MULTIPLY: return "SCALAR_MULTIPLY";
        case OpType::SILU: return "SILU";
        case OpType::GELU: return "GELU";
        case OpType::SAMPLE: return "SAMPLE";
        case OpType::INDEX: return "INDEX";
        case OpType::QUANTIZE_ACTIVATIONS: return "QUANTIZE_ACTIVATIONS";
        default: return "OP";
    }
}
}  // namespace

BufferDesc::BufferDesc(const std::vector<size_t>& s, Precision p) : shape(s), precision(p) {
    total_size = prod(s);
    byte_size = PrecisionTraits::packed_size_of(p, total_size);
}

CactusGraph::CactusGraph() {
    cudaStream_t s = nullptr;
    ck(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "graph stream");
    stream_ = s;
}

CactusGraph::~CactusGraph() {
    try {
        hard_reset();
    } catch (...) {
    }
    for (void* p : scratch_) cudaFree(p);
    if (stream_) cudaStreamDestroy(static_cast<cudaStream_t>(stream_));
}

size_t CactusGraph::add_node(OpType op_type, const std::vector<size_t>& inputs, const std::vector<size_t>& output_shape,
                             const OpParams& params) {
    for (size_t id : inputs)
        if (!node_index_map_.count(id)) throw std::invalid_argument("unknown input node id " + std::to_string(id));
    auto node = std::make_unique<GraphNode>(next_node_id_, op_type);
    node->input_ids = inputs;
    node->params = params;
    std::vector<size_t> shape = output_shape;
    if (shape.empty() && !inputs.empty()) shape = nodes_[node_index_map_[inputs[0]]]->output_buffer.shape;
    Precision prec = params.output_precision;
    // the reference's rule (an INT8 request inherits the first input's precision) would label
    // a QUANTIZE_ACTIVATIONS node FP16, so a later matmul could not see it as pre-quantized;
    // that node keeps INT8 here
    if (op_type != OpType::PRECISION_CAST && op_type != OpType::QUANTIZE_ACTIVATIONS && prec == Precision::INT8 &&
        !inputs.empty())
        prec = nodes_[node_index_map_[inputs[0]]]->output_buffer.precision;
    node->output_buffer = BufferDesc(shape, prec);
    const size_t id = next_node_id_++;
    node_index_map_[id] = nodes_.size();
    nodes_.push_back(std::move(node));
    return id;
}

const BufferDesc& CactusGraph::get_output_buffer(size_t node_id) const {
    return nodes_[node_index_map_.at(node_id)]->output_buffer;
}

size_t CactusGraph::input(const std::vector<size_t>& shape, Precision precision) {
    OpParams p;
    p.output_precision = precision;
    return add_node(OpType::INPUT, {}, shape, p);
}

size_t CactusGraph::quantize_activations(size_t in) {
    if (get_output_buffer(in).precision != Precision::FP16)
        throw std::invalid_argument("quantize_activations requires FP16 input");
    OpParams p;
    p.output_precision = Precision::INT8;
    return add_node(OpType::QUANTIZE_ACTIVATIONS, {in}, get_output_buffer(in).shape, p);
}

static void same_shape(const BufferDesc& a, const BufferDesc& b) {
    if (a.shape != b.shape) throw std::invalid_argument("broadcasting is not supported by the B200 backend");
}
size_t CactusGraph::add(size_t a, size_t b) {
    same_shape(get_output_buffer(a), get_output_buffer(b));
    return add_node(OpType::ADD, {a, b}, get_output_buffer(a).shape);
}
size_t CactusGraph::add_clipped(size_t a, size_t b) {
    same_shape(get_output_buffer(a), get_output_buffer(b));
    return add_node(OpType::ADD_CLIPPED, {a, b}, get_output_buffer(a).shape);
}
size_t CactusGraph::multiply(size_t a, size_t b) {
    same_shape(get_output_buffer(a), get_output_buffer(b));
    return add_node(OpType::MULTIPLY, {a, b}, get_output_buffer(a).shape);
}
size_t CactusGraph::scalar_multiply(size_t in, float value) {
    OpParams p;
    p.scalar = value;
    return add_node(OpType::SCALAR_MULTIPLY, {in}, {}, p);
}
size_t CactusGraph::silu(size_t in) { return add_node(OpType::SILU, {in}, {}); }
size_t CactusGraph::gelu(size_t in) { return add_node(OpType::GELU, {in}, {}); }

// graph_builder.cpp:61-81
size_t CactusGraph::matmul(size_t a, size_t b, bool pretransposed_rhs, ComputeBackend backend) {
    const auto& l = get_output_buffer(a);
    const auto& r = get_output_buffer(b);
    if (l.shape.size() != 2 || r.shape.size() != 2) throw std::invalid_argument("Matrix multiplication requires 2D tensors");
    const size_t M = l.shape[0], K = l.shape[1];
    const size_t rK = pretransposed_rhs ? r.shape[1] : r.shape[0];
    const size_t N = pretransposed_rhs ? r.shape[0] : r.shape[1];
    if (K != rK) throw std::invalid_argument("Matrix dimensions incompatible for multiplication");
    OpParams p;
    p.pretransposed_rhs = pretransposed_rhs;
    p.backend = backend;
    p.output_precision = Precision::FP16;
    return add_node(OpType::MATMUL, {a, b}, {M, N}, p);
}

size_t CactusGraph::transpose(size_t in, ComputeBackend backend) {
    auto s = get_output_buffer(in).shape;
    if (s.size() != 2) throw std::invalid_argument("transpose supports 2D tensors in the B200 backend");
    std::swap(s[0], s[1]);
    OpParams p;
    p.backend = backend;
    return add_node(OpType::TRANSPOSE, {in}, s, p);
}

size_t CactusGraph::reshape(size_t in, const std::vector<size_t>& new_shape) {
    if (prod(new_shape) != get_output_buffer(in).total_size) throw std::invalid_argument("reshape changes the element count");
    OpParams p;
    p.new_shape = new_shape;
    return add_node(OpType::RESHAPE, {in}, new_shape, p);
}

// graph_builder.cpp:123-159
size_t CactusGraph::index(size_t in, size_t index_value, int dim) {
    const auto& b = get_output_buffer(in);
    if (b.shape.empty()) throw std::invalid_argument("Cannot index a scalar tensor");
    int d = dim < 0 ? dim + (int)b.shape.size() : dim;
    if (d < 0 || (size_t)d >= b.shape.size()) throw std::invalid_argument("Index dimension out of bounds");
    if (index_value >= b.shape[d])
        throw std::invalid_argument("Index value " + std::to_string(index_value) + " out of bounds for dimension " +
                                    std::to_string(d) + " with size " + std::to_string(b.shape[d]));
    if (d != 0) throw std::invalid_argument("index supports dim 0 in the B200 backend");
    std::vector<size_t> out(b.shape.begin() + 1, b.shape.end());
    if (out.empty()) out = {1};
    OpParams p;
    p.axis = d;
    p.index_value = index_value;
    p.output_precision = b.precision;
    return add_node(OpType::INDEX, {in}, out, p);
}

// graph_io.cpp:25-73: the .weights file is read once and uploaded to HBM
static size_t load_weights_node(CactusGraph& g, const std::string& filename) {
    cb::eng::HostTensor t = cb::eng::read_weights_file(filename);
    Precision p = t.prec == cb::eng::kInt8 ? Precision::INT8
                : t.prec == cb::eng::kInt4 ? Precision::INT4
                : t.prec == cb::eng::kFp16 ? Precision::FP16 : Precision::FP32;
    // INT4 files are presented as INT8 nodes whose data stays packed (effective_precision,
    // graph.h:526-528); the matmul dispatches on the packed flag
    const size_t id = g.input(t.shape, p == Precision::INT4 ? Precision::INT8 : p);
    auto& b = g.nodes_[g.node_index_map_.at(id)]->output_buffer;
    void* d = nullptr;
    ck(cudaMalloc(&d, t.data.size() ? t.data.size() : 16), "weights");
    ck(cudaMemcpy(d, t.data.data(), t.data.size(), cudaMemcpyHostToDevice), "weights");
    b.device_data = d;
    b.owns_data = true;
    b.packed_int4 = p == Precision::INT4;
    if (!t.scales.empty()) {
        void* s = nullptr;
        ck(cudaMalloc(&s, t.scales.size() * 2), "scales");
        ck(cudaMemcpy(s, t.scales.data(), t.scales.size() * 2, cudaMemcpyHostToDevice), "scales");
        b.scales_data = s;
        b.owns_scales = true;
        b.group_size = t.group_size;
        b.num_groups = t.num_groups;
    }
    return id;
}

size_t CactusGraph::mmap_weights(const std::string& filename) {
    auto it = weight_cache_.find(filename);
    if (it != weight_cache_.end()) return it->second;
    const size_t id = load_weights_node(*this, filename);
    weight_cache_[filename] = id;
    return id;
}

size_t CactusGraph::mmap_embeddings(const std::string& filename) {
    const size_t id = load_weights_node(*this, filename);
    if (get_output_buffer(id).shape.size() != 2)
        throw std::runtime_error("Memory-mapped embeddings must be 2D [vocab_size, embedding_dim]");
    return id;
}

void CactusGraph::set_grouped_scales(size_t node_id, size_t group_size, size_t num_groups, void* scales_ptr) {
    auto it = node_index_map_.find(node_id);
    if (it == node_index_map_.end()) return;
    auto& b = nodes_[it->second]->output_buffer;
    const size_t rows = b.shape.empty() ? 0 : b.total_size / b.shape.back();
    const size_t bytes = rows * num_groups * 2;
    if (is_device_ptr(scales_ptr)) {
        b.scales_data = scales_ptr;
        b.owns_scales = false;
    } else {
        void* d = nullptr;
        ck(cudaMalloc(&d, bytes ? bytes : 16), "scales");
        ck(cudaMemcpy(d, scales_ptr, bytes, cudaMemcpyHostToDevice), "scales");
        b.scales_data = d;
        b.owns_scales = true;
    }
    b.group_size = group_size;
    b.num_groups = num_groups;
}

size_t CactusGraph::embedding(const std::string& filename, size_t indices) {
    const size_t table = mmap_embeddings(filename);
    return embedding(table, indices);
}

size_t CactusGraph::embedding(size_t table, size_t indices) {
    const auto& t = get_output_buffer(table);
    if (t.shape.size() != 2) throw std::runtime_error("Embedding file must contain 2D tensor [vocab_size, hidden_dim]");
    std::vector<size_t> out = get_output_buffer(indices).shape;
    out.push_back(t.shape[1]);
    OpParams p;
    p.output_precision = Precision::FP16;
    return add_node(OpType::EMBEDDING, {table, indices}, out, p);
}

size_t CactusGraph::layernorm(size_t in, size_t weight, size_t bias, float epsilon) {
    OpParams p;
    p.epsilon = epsilon;
    return add_node(OpType::LAYERNORM, {in, weight, bias}, {}, p);
}

size_t CactusGraph::conv1d_causal(size_t in, size_t weight, size_t, size_t dilation) {
    OpParams p;
    p.dilation = dilation;
    return add_node(OpType::CONV1D_CAUSAL, {in, weight}, {}, p);
}

size_t CactusGraph::conv1d_k3(size_t in, size_t weight, size_t stride) {  // graph_builder.cpp:323-345
    const BufferDesc& x = get_output_buffer(in);
    const BufferDesc& w = get_output_buffer(weight);
    if (x.shape.size() != 3) throw std::runtime_error("conv1d_k3 expects N,C,L");
    if (w.shape.size() != 3) throw std::runtime_error("weight must be [C_out,C_in,3]");
    if (w.shape[1] != x.shape[1]) throw std::runtime_error("C_in mismatch in conv1d_k3");
    if (w.shape[2] != 3) throw std::runtime_error("K=3 expected in conv1d_k3");
    if (stride == 0) throw std::runtime_error("conv1d_k3: stride must be >= 1");
    OpParams p;
    p.stride = stride;
    p.output_precision = x.precision;
    return add_node(OpType::CONV1D_K3, {in, weight}, {x.shape[0], w.shape[0], (x.shape[2] - 1) / stride + 1}, p);
}

size_t CactusGraph::rms_norm(size_t in, size_t weight, float epsilon) {
    OpParams p;
    p.epsilon = epsilon;
    return add_node(OpType::RMS_NORM, {in, weight}, {}, p);
}

size_t CactusGraph::rope(size_t in, float theta, size_t position_offset, ComputeBackend backend) {
    OpParams p;
    p.theta = theta;
    p.position_offset = position_offset;
    p.backend = backend;
    return add_node(OpType::ROPE, {in}, {}, p);
}

size_t CactusGraph::softmax(size_t in, int axis) {
    OpParams p;
    p.axis = axis;
    return add_node(OpType::SOFTMAX, {in}, {}, p);
}

size_t CactusGraph::attention(size_t q, size_t k, size_t v, float scale, bool is_causal, ComputeBackend backend) {
    OpParams p;
    p.scale = scale;
    p.is_causal = is_causal;
    p.backend = backend;
    return add_node(OpType::ATTENTION, {q, k, v}, {}, p);
}
size_t CactusGraph::attention(size_t q, size_t k, size_t v, float scale, size_t position_offset,
                              ComputeBackend backend) {
    OpParams p;
    p.scale = scale;
    p.position_offset = position_offset;
    p.backend = backend;
    return add_node(OpType::ATTENTION, {q, k, v}, {}, p);
}
size_t CactusGraph::attention(size_t q, size_t k, size_t v, float scale, size_t position_offset, size_t window_size,
                              ComputeBackend backend) {
    OpParams p;
    p.scale = scale;
    p.position_offset = position_offset;
    p.window_size = window_size;
    p.backend = backend;
    return add_node(OpType::ATTENTION, {q, k, v}, {}, p);
}

size_t CactusGraph::attention_int8_hybrid(size_t q, size_t k_new, size_t v_new, float scale, size_t position_offset,
                                          const int8_t* cached_keys, const int8_t* cached_values,
                                          const float* k_scales, const float* v_scales, size_t cache_len,
                                          size_t num_kv_heads, size_t head_dim) {
    OpParams p;
    p.scale = scale;
    p.position_offset = position_offset;
    p.cached_keys_int8 = cached_keys;
    p.cached_values_int8 = cached_values;
    p.cached_k_scales = k_scales;
    p.cached_v_scales = v_scales;
    p.cache_seq_len = cache_len;
    p.num_kv_heads = num_kv_heads;
    p.head_dim = head_dim;
    return add_node(OpType::ATTENTION_INT8_HYBRID, {q, k_new, v_new}, get_output_buffer(q).shape, p);
}

size_t CactusGraph::sample(size_t logits, float temperature, float top_p, size_t top_k,
                           const std::unordered_map<uint32_t, float>&) {
    if (get_output_buffer(logits).shape.empty()) throw std::runtime_error("Sample requires non-empty logits tensor");
    OpParams p;
    p.temperature = temperature;
    p.top_p = top_p;
    p.top_k = top_k;
    p.random_seed = (size_t)std::chrono::high_resolution_clock::now().time_since_epoch().count();
    p.output_precision = Precision::FP32;  // 4-byte slot holding a uint32 token id
    return add_node(OpType::SAMPLE, {logits}, {1}, p);
}

// graph_execute.cpp:197-221
void CactusGraph::set_input(size_t node_id, const void* data, Precision) {
    auto& n = *nodes_[node_index_map_.at(node_id)];
    if (n.op_type != OpType::INPUT) throw std::invalid_argument("Can only set data on input nodes");
    if (n.output_buffer.is_packed_int4())
        throw std::invalid_argument("Cannot use set_input on packed INT4 buffer - use set_external_input instead");
    void* d = ensure_device(n.output_buffer);
    ck(cudaMemcpyAsync(d, data, n.output_buffer.byte_size, cudaMemcpyHostToDevice,
                       static_cast<cudaStream_t>(stream_)),
       "set_input");
    ck(cudaStreamSynchronize(static_cast<cudaStream_t>(stream_)), "set_input");
}

void CactusGraph::set_external_input(size_t node_id, void* data, Precision) {
    auto& n = *nodes_[node_index_map_.at(node_id)];
    if (n.op_type != OpType::INPUT) throw std::invalid_argument("Can only set data on input nodes");
    if (is_device_ptr(data)) {
        if (n.output_buffer.owns_data && n.output_buffer.device_data) cudaFree(n.output_buffer.device_data);
        n.output_buffer.device_data = data;
        n.output_buffer.owns_data = false;
    } else {
        void* d = ensure_device(n.output_buffer);
        ck(cudaMemcpy(d, data, n.output_buffer.byte_size, cudaMemcpyHostToDevice), "set_external_input");
    }
}

void* CactusGraph::ensure_device(BufferDesc& b) {
    if (!b.device_data) {
        void* d = nullptr;
        ck(cudaMalloc(&d, b.byte_size ? b.byte_size : 16), "buffer");
        b.device_data = d;
        b.owns_data = true;
    }
    return b.device_data;
}

void* CactusGraph::scratch(size_t bytes) {
    if (scratch_used_ < scratch_.size() && scratch_bytes_[scratch_used_] >= bytes) return scratch_[scratch_used_++];
    void* d = nullptr;
    ck(cudaMalloc(&d, bytes ? bytes : 16), "scratch");
    if (scratch_used_ < scratch_.size()) {
        cudaFree(scratch_[scratch_used_]);
        scratch_[scratch_used_] = d;
        scratch_bytes_[scratch_used_] = bytes;
    } else {
        scratch_.push_back(d);
        scratch_bytes_.push_back(bytes);
    }
    ++scratch_used_;
    return d;
}

void* CactusGraph::get_output(size_t node_id) {
    auto& b = nodes_[node_index_map_.at(node_id)]->output_buffer;
    ensure_device(b);
    ck(cudaStreamSynchronize(static_cast<cudaStream_t>(stream_)), "get_output");
    b.host_mirror.resize(b.byte_size);
    ck(cudaMemcpy(b.host_mirror.data(), b.device_data, b.byte_size, cudaMemcpyDeviceToHost), "get_output");
    return b.host_mirror.data();
}

void CactusGraph::execute(const std::string& profile_file) {
    cudaStream_t st = static_cast<cudaStream_t>(stream_);
    std::ostringstream prof;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (!profile_file.empty()) {
        ck(cudaEventCreate(&e0), "event");
        ck(cudaEventCreate(&e1), "event");
    }
    double total_ms = 0;
    for (auto& np : nodes_) {
        if (np->op_type == OpType::INPUT) continue;
        if (e0) ck(cudaEventRecord(e0, st), "event");
        compute_node(*np);
        if (e0) {
            ck(cudaEventRecord(e1, st), "event");
            ck(cudaEventSynchronize(e1), "event");
            float ms = 0;
            cudaEventElapsedTime(&ms, e0, e1);
            total_ms += ms;
            prof << std::left << std::setw(24) << op_name(np->op_type) << std::fixed << std::setprecision(3) << ms
                 << " ms  [";
            for (size_t i = 0; i < np->output_buffer.shape.size(); ++i)
                prof << (i ? "," : "") << np->output_buffer.shape[i];
            prof << "]\n";
        }
    }
    ck(cudaStreamSynchronize(st), "execute");
    if (e0) {
        prof << "TOTAL " << std::fixed << std::setprecision(3) << total_ms << " ms\n";
        std::ofstream f(profile_file, std::ios::app);
        f << prof.str();
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
    }
}

void CactusGraph::soft_reset() {
    // keeps cached weights (mmap_weights), drops every other node (graph_execute.cpp:640-675)
    std::vector<std::unique_ptr<GraphNode>> keep;
    std::unordered_map<size_t, size_t> keep_map;
    for (auto& np : nodes_) {
        bool cached = false;
        for (auto& kv : weight_cache_)
            if (kv.second == np->id) cached = true;
        if (cached) {
            keep_map[np->id] = keep.size();
            keep.push_back(std::move(np));
        } else if (np) {
            auto& b = np->output_buffer;
            if (b.owns_data && b.device_data) cudaFree(b.device_data);
            if (b.owns_scales && b.scales_data) cudaFree(b.scales_data);
            if (b.activation_scales) cudaFree(b.activation_scales);
        }
    }
    nodes_ = std::move(keep);
    node_index_map_ = std::move(keep_map);
    scratch_used_ = 0;
}

void CactusGraph::hard_reset() {
    cudaStreamSynchronize(static_cast<cudaStream_t>(stream_));
    for (auto& np : nodes_) {
        auto& b = np->output_buffer;
        if (b.owns_data && b.device_data) cudaFree(b.device_data);
        if (b.owns_scales && b.scales_data) cudaFree(b.scales_data);
        if (b.activation_scales) cudaFree(b.activation_scales);
    }
    nodes_.clear();
    node_index_map_.clear();
    weight_cache_.clear();
    next_node_id_ = 0;
    scratch_used_ = 0;
}

// ------------------------------------------------------------------ node executors
void CactusGraph::compute_node(GraphNode& node) {
    cudaStream_t st = static_cast<cudaStream_t>(stream_);
    void* sv = st;
    auto in = [&](int i) -> BufferDesc& { return nodes_[node_index_map_.at(node.input_ids[i])]->output_buffer; };
    BufferDesc& out = node.output_buffer;
    auto u16 = [](void* p) { return static_cast<uint16_t*>(p); };
    auto need = [](const BufferDesc& b, Precision p, const char* what) {
        if (b.precision != p) throw std::runtime_error(what);
        if (!b.device_data) throw std::runtime_error(std::string(what) + ": input has no data");
    };
    switch (node.op_type) {
        case OpType::RESHAPE:
        case OpType::INDEX: {
            BufferDesc& src = in(0);
            if (!src.device_data) throw std::runtime_error("reshape/index of an empty buffer");
            size_t off = 0;
            if (node.op_type == OpType::INDEX)
                off = node.params.index_value * (src.total_size / src.shape[0]) * PrecisionTraits::size_of(src.precision);
            if (out.owns_data && out.device_data) cudaFree(out.device_data);
            out.device_data = static_cast<char*>(src.device_data) + off;  // a view, as the reference's INDEX dim 0
            out.owns_data = false;
            out.precision = src.precision;
            return;
        }
        default:
            break;
    }
    void* o = ensure_device(out);
    switch (node.op_type) {
        case OpType::QUANTIZE_ACTIVATIONS: {
            BufferDesc& x = in(0);
            need(x, Precision::FP16, "QUANTIZE_ACTIVATIONS requires FP16 input");
            const size_t K = x.shape.back(), M = x.total_size / K;
            if (!out.activation_scales) ck(cudaMalloc(reinterpret_cast<void**>(&out.activation_scales), M * 4), "scales");
            out.num_rows_for_activation_scales = M;
            kck(cactus_cuda_quantize_activations(u16(x.device_data), static_cast<int8_t*>(o), out.activation_scales,
                                                 M, K, sv), "quantize_activations");
            break;
        }
        case OpType::MATMUL: {  // compute_matmul_node, graph_ops_nn.cpp:129-231
            BufferDesc& l = in(0);
            BufferDesc& r = in(1);
            const size_t M = l.shape[0], K = l.shape[1];
            const size_t N = node.params.pretransposed_rhs ? r.shape[0] : r.shape[1];
            out.precision = Precision::FP16;
            const bool preq = l.precision == Precision::INT8 && l.has_activation_scales();
            if (r.is_packed_int4() || r.is_grouped_int8()) {
                if (!node.params.pretransposed_rhs)
                    throw std::runtime_error(r.is_packed_int4() ? "INT4 matmul requires pretransposed weights"
                                                                : "Group-wise INT8 matmul requires pretransposed weights");
                if (preq) {
                    kck(r.is_packed_int4()
                            ? cactus_cuda_matmul_int4(static_cast<int8_t*>(l.device_data), l.activation_scales,
                                                      static_cast<uint8_t*>(r.device_data), u16(r.scales_data), u16(o),
                                                      M, K, N, r.group_size, sv)
                            : cactus_cuda_matmul_int8(static_cast<int8_t*>(l.device_data), l.activation_scales,
                                                      static_cast<int8_t*>(r.device_data), u16(r.scales_data), u16(o),
                                                      M, K, N, r.group_size, sv),
                        "matmul");
                } else if (l.precision == Precision::FP16) {
                    kck(r.is_packed_int4()
                            ? cactus_cuda_linear_int4(u16(l.device_data), static_cast<uint8_t*>(r.device_data),
                                                      u16(r.scales_data), u16(o), M, K, N, r.group_size, sv)
                            : cactus_cuda_linear_int8(u16(l.device_data), static_cast<int8_t*>(r.device_data),
                                                      u16(r.scales_data), u16(o), M, K, N, r.group_size, sv),
                        "matmul");
                } else {
                    throw std::runtime_error("INT8 matmul requires INT8 (pre-quantized) or FP16 activations");
                }
            } else {
                if (l.precision != Precision::FP16) throw std::runtime_error("FP16 matmul requires FP16 activations");
                if (r.precision != Precision::FP16)
                    throw std::runtime_error("INT8 weights need group scales (set_grouped_scales) in the B200 backend");
                const uint16_t* bt = u16(r.device_data);
                if (!node.params.pretransposed_rhs) {  // transpose [K,N] -> [N,K] first (graph_ops_nn.cpp:220-229)
                    void* t = scratch(K * N * 2);
                    kck(cactus_cuda_transpose_2d_f16(u16(r.device_data), u16(t), K, N, sv), "transpose");
                    bt = u16(t);
                }
                kck(cactus_cuda_matmul_f16(u16(l.device_data), bt, u16(o), M, K, N, sv), "matmul_f16");
            }
            break;
        }
        case OpType::TRANSPOSE: {
            BufferDesc& x = in(0);
            need(x, Precision::FP16, "transpose supports FP16");
            kck(cactus_cuda_transpose_2d_f16(u16(x.device_data), u16(o), x.shape[0], x.shape[1], sv), "transpose");
            break;
        }
        case OpType::ADD:
        case OpType::ADD_CLIPPED:
        case OpType::MULTIPLY: {
            BufferDesc& a = in(0);
            BufferDesc& b = in(1);
            need(a, Precision::FP16, "binary ops support FP16");
            need(b, Precision::FP16, "binary ops support FP16");
            const auto fn = node.op_type == OpType::ADD ? cactus_cuda_add_f16
                          : node.op_type == OpType::ADD_CLIPPED ? cactus_cuda_add_f16_clipped : cactus_cuda_multiply_f16;
            kck(fn(u16(a.device_data), u16(b.device_data), u16(o), a.total_size, sv), "binary");
            break;
        }
        case OpType::SCALAR_MULTIPLY: {
            BufferDesc& x = in(0);
            need(x, Precision::FP16, "scalar ops support FP16");
            kck(cactus_cuda_scalar_multiply_f16(u16(x.device_data), u16(o), x.total_size, node.params.scalar, sv),
                "scalar_multiply");
            break;
        }
        case OpType::SILU:
        case OpType::GELU: {
            BufferDesc& x = in(0);
            need(x, Precision::FP16, "activations support FP16");
            kck(node.op_type == OpType::SILU ? cactus_cuda_silu_f16(u16(x.device_data), u16(o), x.total_size, sv)
                                             : cactus_cuda_gelu_f16(u16(x.device_data), u16(o), x.total_size, sv),
                "activation");
            break;
        }
        case OpType::RMS_NORM: {  // graph_ops_nn.cpp:233-253
            BufferDesc& x = in(0);
            BufferDesc& w = in(1);
            if (x.shape.size() != 2)
                throw std::runtime_error("RMS normalization requires 2D input tensor [batch_size, dims], got " +
                                         std::to_string(x.shape.size()) + "D tensor");
            need(x, Precision::FP16, "RMS normalization only supports FP16 precision");
            kck(cactus_cuda_rms_norm_f16(u16(x.device_data), u16(w.device_data), u16(o), x.shape[0], x.shape[1],
                                         node.params.epsilon, sv), "rms_norm");
            break;
        }
        case OpType::LAYERNORM: {  // graph_ops_nn.cpp:373-457
            BufferDesc& x = in(0);
            BufferDesc& w = in(1);
            BufferDesc& b = in(2);
            if (x.shape.empty()) throw std::runtime_error("LayerNorm requires non-empty input tensor");
            need(x, Precision::FP16, "LayerNorm on the B200 backend supports FP16 input");
            need(w, Precision::FP16, "LayerNorm on the B200 backend supports FP16 weight");
            need(b, Precision::FP16, "LayerNorm on the B200 backend supports FP16 bias");
            const size_t F = x.shape.back();
            kck(cactus_cuda_layernorm_f16(u16(x.device_data), u16(w.device_data), u16(b.device_data), u16(o),
                                          x.total_size / F, F, node.params.epsilon, sv),
                "layernorm");
            break;
        }
        case OpType::CONV1D_CAUSAL: {  // graph_ops_nn.cpp:459-530
            BufferDesc& x = in(0);
            BufferDesc& w = in(1);
            if (x.shape.size() != 3) throw std::runtime_error("Causal conv requires 3D input [batch, seq_len, in_channels]");
            if (w.shape.size() != 3) throw std::runtime_error("Weight must be 3D");
            if (w.shape[1] != 1 || w.shape[0] != x.shape[2])
                throw std::runtime_error("Only depthwise causal convolution is supported currently");
            if (node.params.dilation < 1) throw std::runtime_error("dilation must be >= 1");
            need(x, Precision::FP16, "Depthwise causal conv on the B200 backend supports FP16 input");
            need(w, Precision::FP16, "Depthwise causal conv on the B200 backend supports FP16 weights");
            kck(cactus_cuda_conv1d_causal_depthwise_f16(u16(x.device_data), u16(w.device_data), u16(o), x.shape[0],
                                                        x.shape[1], x.shape[2], w.shape[2], node.params.dilation, sv),
                "conv1d_causal");
            break;
        }
        case OpType::CONV1D_K3: {  // graph_ops_nn.cpp:532-580
            BufferDesc& x = in(0);
            BufferDesc& w = in(1);
            need(x, Precision::FP16, "Conv1d_k3 on the B200 backend supports FP16 input");
            need(w, Precision::FP16, "Conv1d_k3 on the B200 backend supports FP16 weights");
            kck(cactus_cuda_conv1d_f16_k3(u16(x.device_data), u16(w.device_data), u16(o), x.shape[0], x.shape[2],
                                          x.shape[1], w.shape[0], node.params.stride, sv),
                "conv1d_k3");
            break;
        }
        case OpType::ROPE: {  // graph_ops_nn.cpp:255-282
            BufferDesc& x = in(0);
            if (x.shape.size() < 4)
                throw std::runtime_error("RoPE operation requires 4D tensor with shape [batch, seq_len, num_heads, head_dim], got " +
                                         std::to_string(x.shape.size()) + "D tensor");
            need(x, Precision::FP16, "RoPE operation only supports FP16 precision");
            kck(cactus_cuda_rope_f16(u16(x.device_data), u16(o), x.shape[0], x.shape[1], x.shape[2], x.shape[3],
                                     node.params.position_offset, node.params.theta, sv), "rope");
            break;
        }
        case OpType::SOFTMAX: {
            BufferDesc& x = in(0);
            if (x.shape.size() < 2)
                throw std::runtime_error("Softmax operation requires at least 2D tensor, got " +
                                         std::to_string(x.shape.size()) + "D tensor");
            need(x, Precision::FP16, "Softmax operation only supports FP16 precision");
            const size_t V = x.shape.back();
            kck(cactus_cuda_softmax_f16(u16(x.device_data), u16(o), x.total_size / V, V, sv), "softmax");
            break;
        }
        case OpType::ATTENTION: {  // graph_ops_nn.cpp:306-338
            BufferDesc& q = in(0);
            BufferDesc& k = in(1);
            BufferDesc& v = in(2);
            if (q.shape.size() < 4)
                throw std::runtime_error("Attention operation requires 4D tensors [batch, seq_len, num_heads, head_dim], got " +
                                         std::to_string(q.shape.size()) + "D tensor");
            need(q, Precision::FP16, "Attention operation only supports FP16 precision");
            kck(cactus_cuda_attention_f16(u16(q.device_data), u16(k.device_data), u16(v.device_data), u16(o),
                                          q.shape[0], q.shape[1], k.shape[1], q.shape[2], k.shape[2], q.shape[3],
                                          node.params.scale, node.params.position_offset, node.params.window_size,
                                          node.params.is_causal ? 1 : 0, sv), "attention");
            break;
        }
        case OpType::ATTENTION_INT8_HYBRID: {  // graph_ops_nn.cpp:340-371
            BufferDesc& q = in(0);
            BufferDesc& kn = in(1);
            BufferDesc& vn = in(2);
            if (q.shape.size() < 4) throw std::runtime_error("ATTENTION_INT8_HYBRID requires 4D query tensor");
            kck(cactus_cuda_attention_hybrid_int8_fp16(
                    u16(q.device_data), node.params.cached_keys_int8, node.params.cached_values_int8,
                    node.params.cached_k_scales, node.params.cached_v_scales, u16(kn.device_data), u16(vn.device_data),
                    u16(o), q.shape[0], q.shape[1], node.params.cache_seq_len, kn.shape[1], q.shape[2],
                    node.params.num_kv_heads, node.params.head_dim, node.params.scale, node.params.position_offset, 1,
                    128, sv), "attention_int8_hybrid");
            break;
        }
        case OpType::EMBEDDING: {  // graph_ops_tensor.cpp:226-331 (indices as FP32 or INT8 values)
            BufferDesc& t = in(0);
            BufferDesc& idx = in(1);
            const size_t n = idx.total_size, hidden = t.shape[1];
            std::vector<uint32_t> ids(n);
            if (!idx.device_data) throw std::runtime_error("embedding indices have no data");
            if (idx.precision == Precision::FP32) {
                std::vector<float> f(n);
                ck(cudaMemcpy(f.data(), idx.device_data, n * 4, cudaMemcpyDeviceToHost), "indices");
                for (size_t i = 0; i < n; ++i) ids[i] = (uint32_t)f[i];
            } else {
                std::vector<int8_t> q(n);
                ck(cudaMemcpy(q.data(), idx.device_data, n, cudaMemcpyDeviceToHost), "indices");
                for (size_t i = 0; i < n; ++i) ids[i] = (uint32_t)(size_t)q[i];
            }
            for (uint32_t v : ids)
                if (v >= t.shape[0])
                    throw std::runtime_error("Embedding index out of bounds: " + std::to_string(v) + " >= " +
                                             std::to_string(t.shape[0]));
            uint32_t* d_ids = static_cast<uint32_t*>(scratch(n * 4));
            ck(cudaMemcpyAsync(d_ids, ids.data(), n * 4, cudaMemcpyHostToDevice, st), "indices");
            out.precision = Precision::FP16;
            if (t.precision == Precision::FP16) {
                kck(cactus_cuda_embedding_f16(u16(t.device_data), t.shape[0], hidden, d_ids, n, u16(o), sv), "embedding");
            } else if (t.is_packed_int4()) {
                // the reference unpacks INT4 to INT8 on load (graph_io.cpp:435-455)
                int8_t* un = static_cast<int8_t*>(scratch(t.shape[0] * hidden));
                kck(cactus_cuda_unpack_int4_to_int8(static_cast<uint8_t*>(t.device_data), un, t.shape[0] * hidden, sv),
                    "unpack");
                kck(cactus_cuda_embedding_int8(un, u16(t.scales_data), t.group_size, t.shape[0], hidden, d_ids, n, u16(o),
                                               sv), "embedding");
            } else if (t.is_grouped_int8()) {
                kck(cactus_cuda_embedding_int8(static_cast<int8_t*>(t.device_data), u16(t.scales_data), t.group_size,
                                               t.shape[0], hidden, d_ids, n, u16(o), sv), "embedding");
            } else if (t.precision == Precision::INT8) {
                // ungrouped INT8 converts each value to fp16: one group per row with scale 1.0
                std::vector<uint16_t> ones(t.shape[0], 0x3C00);
                uint16_t* d_ones = static_cast<uint16_t*>(scratch(t.shape[0] * 2));
                ck(cudaMemcpyAsync(d_ones, ones.data(), ones.size() * 2, cudaMemcpyHostToDevice, st), "scales");
                kck(cactus_cuda_embedding_int8(static_cast<int8_t*>(t.device_data), d_ones, hidden, t.shape[0], hidden,
                                               d_ids, n, u16(o), sv), "embedding");
                ck(cudaStreamSynchronize(st), "embedding");
            } else {
                throw std::runtime_error("Embedding only supports INT8 and FP16 precision");
            }
            ck(cudaStreamSynchronize(st), "embedding");
            break;
        }
        case OpType::SAMPLE: {  // graph_ops_sample.cpp:8-39 (last row)
            BufferDesc& lg = in(0);
            if (lg.shape.size() != 2) throw std::runtime_error("Sample expects 2D logits tensor [seq_len, vocab_size]");
            need(lg, Precision::FP16, "sample supports FP16 logits");
            const size_t rows = lg.shape[0], V = lg.shape[1];
            const float t = node.params.temperature, tp = node.params.top_p;
            const size_t tk = node.params.top_k;
            if (t == 0.0f && tp <= 0.0f && tk == 0) {
                kck(cactus_cuda_argmax_f16(u16(lg.device_data), rows, V, static_cast<uint32_t*>(o), sv), "sample");
            } else {
                std::mt19937 gen((uint32_t)node.params.random_seed);
                std::uniform_real_distribution<float> dist(0.0f, 1.0f);
                uint32_t* hist = static_cast<uint32_t*>(scratch(128 * 4));
                if (!sample_history_.empty())
                    ck(cudaMemcpyAsync(hist, sample_history_.data(), sample_history_.size() * 4,
                                       cudaMemcpyHostToDevice, st), "history");
                kck(cactus_cuda_sample_f16(u16(lg.device_data), rows, V, t, tp, tk, dist(gen), hist,
                                           sample_history_.size(), u16(scratch(V * 2)), static_cast<uint32_t*>(o), sv),
                    "sample");
                uint32_t tok = 0;
                ck(cudaMemcpyAsync(&tok, o, 4, cudaMemcpyDeviceToHost, st), "sample");
                ck(cudaStreamSynchronize(st), "sample");
                sample_history_.push_back(tok);
                if (sample_history_.size() > 128) sample_history_.erase(sample_history_.begin());
            }
            break;
        }
        default:
            throw std::runtime_error(std::string("operation not supported by the B200 backend: ") + op_name(node.op_type));
    }
}
