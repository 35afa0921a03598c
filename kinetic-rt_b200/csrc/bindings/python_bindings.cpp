// pybind11 module python.kinetic_rt._core (and _core_mock, the same runtime
// over the host-only CUDA test double).
//
// Class and method names, argument names and error types follow the
// reference's bindings/python_bindings.cpp:219-447 so existing callers work
// unchanged: DataType, TensorDescriptor (zero-copy validation),
// GraphWrapper, HardwareMismatchError, KernelLaunchDescriptor, AOTEngine,
// Serializer, Communicator, HardwareRouter, InferenceQueue, InferenceWorker.
// Additions: BlockManager, descriptor fields of the paged path, and the
// peer-buffer and fused GEMM + allreduce methods of Communicator.
#include <pybind11/pybind11.h>
#include <pybind11/functional.h>
#include <pybind11/stl.h>

#include <chrono>
#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <string>
#include <vector>

#include "AOTEngine.h"
#include "AsyncAPI.h"
#include "BlockManager.h"
#include "Communicator.h"
#include "GraphWrapper.h"
#include "RequestContext.h"
#include "Router.h"

namespace py = pybind11;

#define KRT_STR2(x) #x
#define KRT_STR(x) KRT_STR2(x)

enum class DataType : int { UNKNOWN = 0, FLOAT32 = 1, FLOAT16 = 2, BFLOAT16 = 3, INT32 = 4, INT64 = 5, INT8 = 6, BOOL = 7 };

static const char* dtype_name(DataType t) {
  switch (t) {
    case DataType::FLOAT32: return "float32";
    case DataType::FLOAT16: return "float16";
    case DataType::BFLOAT16: return "bfloat16";
    case DataType::INT32: return "int32";
    case DataType::INT64: return "int64";
    case DataType::INT8: return "int8";
    case DataType::BOOL: return "bool";
    default: return "unknown";
  }
}

static size_t dtype_size(DataType t) {
  switch (t) {
    case DataType::FLOAT32: case DataType::INT32: return 4;
    case DataType::FLOAT16: case DataType::BFLOAT16: return 2;
    case DataType::INT64: return 8;
    case DataType::INT8: case DataType::BOOL: return 1;
    default: return 0;
  }
}

struct TensorDescriptor {
  uintptr_t data_ptr = 0;
  std::vector<int64_t> shape;
  std::vector<int64_t> strides;
  DataType dtype = DataType::UNKNOWN;
  size_t byte_size = 0;
};

static std::string join(const std::vector<int64_t>& v) {
  std::string s = "[";
  for (size_t i = 0; i < v.size(); ++i) s += (i ? "," : "") + std::to_string(v[i]);
  return s + "]";
}

static size_t numel_of(const TensorDescriptor& d) {
  size_t n = 1;
  for (int64_t s : d.shape) {
    if (s <= 0) return 0;
    if (n > SIZE_MAX / static_cast<size_t>(s)) throw std::invalid_argument("TensorDescriptor numel overflows size_t.");
    n *= static_cast<size_t>(s);
  }
  return n;
}

static bool c_contiguous(const TensorDescriptor& d) {
  if (d.shape.empty()) return true;
  if (d.strides.size() != d.shape.size()) return false;
  int64_t expect = 1;
  for (size_t i = d.shape.size(); i-- > 0;) {
    if (d.shape[i] != 1 && d.strides[i] != expect) return false;
    if (d.shape[i] > 0 && expect > INT64_MAX / d.shape[i]) return false;
    expect *= d.shape[i];
  }
  return true;
}

// Zero-copy contract of the reference (bindings/python_bindings.cpp:106-171).
static void validate_descriptor(const TensorDescriptor& d, const std::string& name) {
  const std::string who = "TensorDescriptor('" + name + "')";
  if (d.data_ptr == 0)
    throw std::invalid_argument(who + " has a null data_ptr; the underlying storage has not been allocated.");
  if (d.dtype == DataType::UNKNOWN)
    throw std::invalid_argument(who + " has dtype=UNKNOWN; the Python side failed to map the torch dtype to a "
                                      "supported DataType enum value.");
  if (d.shape.empty()) {
    if (d.byte_size != dtype_size(d.dtype))
      throw std::invalid_argument(who + " (0-d scalar) byte_size=" + std::to_string(d.byte_size) +
                                  " does not match element_size=" + std::to_string(dtype_size(d.dtype)) + " for " +
                                  dtype_name(d.dtype) + ".");
    return;
  }
  if (d.strides.size() != d.shape.size())
    throw std::invalid_argument(who + " strides rank (" + std::to_string(d.strides.size()) + ") != shape rank (" +
                                std::to_string(d.shape.size()) + ").");
  const size_t n = numel_of(d);
  if (n == 0)
    throw std::invalid_argument(who + " has zero numel; empty tensors cannot be forwarded across the zero-copy boundary.");
  if (d.byte_size != n * dtype_size(d.dtype))
    throw std::invalid_argument(who + " byte_size=" + std::to_string(d.byte_size) + " does not match numel*element_size=" +
                                std::to_string(n * dtype_size(d.dtype)) + " (" + std::to_string(n) + " * " +
                                std::to_string(dtype_size(d.dtype)) + " for " + dtype_name(d.dtype) + ").");
  if (!c_contiguous(d))
    throw std::invalid_argument(who + " is not C-contiguous: shape=" + join(d.shape) + " strides=" + join(d.strides) +
                                ". Sliced or transposed tensors with non-unit strides are explicitly blocked; call "
                                "tensor.contiguous() before invoking the runtime.");
}

static TensorDescriptor descriptor_from_tensor(py::object t, const std::string& name) {
  TensorDescriptor d;
  d.data_ptr = t.attr("data_ptr")().cast<uintptr_t>();
  d.shape = t.attr("shape").cast<std::vector<int64_t>>();
  d.strides = t.attr("stride")().cast<std::vector<int64_t>>();
  const int64_t off = t.attr("storage_offset")().cast<int64_t>();
  if (off != 0)
    throw std::invalid_argument("torch.Tensor('" + name + "') has storage_offset=" + std::to_string(off) +
                                " (elements). The zero-copy boundary requires storage_offset == 0; call tensor.clone() "
                                "(or tensor.contiguous().clone()) to materialize a dense tensor before invoking the runtime.");
  py::module torch = py::module::import("torch");
  py::object dt = t.attr("dtype");
  const std::pair<const char*, DataType> table[] = {
      {"float32", DataType::FLOAT32}, {"float16", DataType::FLOAT16}, {"bfloat16", DataType::BFLOAT16},
      {"int32", DataType::INT32},     {"int64", DataType::INT64},     {"int8", DataType::INT8},
      {"bool", DataType::BOOL}};
  for (const auto& e : table)
    if (dt.equal(torch.attr(e.first))) d.dtype = e.second;
  if (d.dtype == DataType::UNKNOWN)
    throw std::invalid_argument("torch.Tensor('" + name + "') has unsupported dtype '" + std::string(py::str(dt)) +
                                "'. Supported: float32, float16, bfloat16, int32, int64, int8, bool.");
  d.byte_size = t.attr("numel")().cast<size_t>() * dtype_size(d.dtype);
  if (t.attr("untyped_storage")().attr("nbytes")().cast<size_t>() < d.byte_size)
    throw std::invalid_argument("torch.Tensor('" + name + "') logical view exceeds actual physical storage allocation bounds.");
  validate_descriptor(d, name);
  return d;
}

// A stream argument: a raw handle (int) or an object with `cuda_stream`.
static uintptr_t stream_of(const py::object& o) {
  if (o.is_none()) return 0;
  if (py::hasattr(o, "cuda_stream")) return o.attr("cuda_stream").cast<uintptr_t>();
  return o.cast<uintptr_t>();
}

PYBIND11_MODULE(KRT_MODULE_NAME, m) {
  m.doc() = "Kinetic-RT B200 runtime: AOT engine, CUDA-graph wrapper, paged KV pool, NVLink communicator";
#if defined(KRT_MOCK_CUDA)
  m.attr("MOCK_CUDA") = true;
  m.def("fake_cuda_state", [] {
    const FakeCudaState& s = fake_cuda_state();
    py::dict d;
    d["stream_begin_capture"] = s.stream_begin_capture;
    d["stream_end_capture"] = s.stream_end_capture;
    d["graph_instantiate"] = s.graph_instantiate;
    d["graph_launch"] = s.graph_launch;
    d["graph_exec_destroy"] = s.graph_exec_destroy;
    d["event_record"] = s.event_record;
    d["library_load"] = s.library_load;
    d["kernel_launch"] = s.kernel_launch;
    d["capturing"] = s.capturing;
    return d;
  });
  m.def("reset_fake_cuda_state", [] { fake_cuda_state().reset(); });
#else
  m.attr("MOCK_CUDA") = false;
#endif

  py::enum_<DataType>(m, "DataType", py::module_local())
      .value("UNKNOWN", DataType::UNKNOWN)
      .value("FLOAT32", DataType::FLOAT32)
      .value("FLOAT16", DataType::FLOAT16)
      .value("BFLOAT16", DataType::BFLOAT16)
      .value("INT32", DataType::INT32)
      .value("INT64", DataType::INT64)
      .value("INT8", DataType::INT8)
      .value("BOOL", DataType::BOOL)
      .export_values();

  py::class_<TensorDescriptor>(m, "TensorDescriptor", py::module_local(),
                               "Metadata needed to dereference a tensor's storage from native code (strides in elements).")
      .def(py::init<>())
      .def_readwrite("data_ptr", &TensorDescriptor::data_ptr)
      .def_readwrite("shape", &TensorDescriptor::shape)
      .def_readwrite("strides", &TensorDescriptor::strides)
      .def_readwrite("dtype", &TensorDescriptor::dtype)
      .def_readwrite("byte_size", &TensorDescriptor::byte_size)
      .def_static("from_tensor", &descriptor_from_tensor, py::arg("tensor"), py::arg("name") = "tensor")
      .def("validate", [](const TensorDescriptor& d, const std::string& name) { validate_descriptor(d, name); },
           py::arg("name") = "tensor")
      .def("__repr__", [](const TensorDescriptor& d) {
        char buf[32];
        std::snprintf(buf, sizeof(buf), "%lx", static_cast<unsigned long>(d.data_ptr));
        return std::string("TensorDescriptor(data_ptr=0x") + buf + ", shape=" + join(d.shape) + ", strides=" +
               join(d.strides) + ", dtype=" + dtype_name(d.dtype) + ", byte_size=" + std::to_string(d.byte_size) + ")";
      });

  py::class_<BlockManager>(m, "BlockManager", py::module_local())
      .def(py::init<int, int, int>(), py::arg("num_blocks"), py::arg("tokens_per_block"), py::arg("token_byte_size"))
      .def("allocate_block", &BlockManager::allocate_block)
      .def("free_block", &BlockManager::free_block, py::arg("id"))
      .def("get_pool_ptr", [](const BlockManager& b) { return reinterpret_cast<uintptr_t>(b.get_pool_ptr()); })
      .def("block_ptr", [](const BlockManager& b, int id) { return reinterpret_cast<uintptr_t>(b.block_ptr(id)); },
           py::arg("id"))
      .def_property_readonly("num_blocks", &BlockManager::num_blocks)
      .def_property_readonly("tokens_per_block", &BlockManager::tokens_per_block)
      .def_property_readonly("token_byte_size", &BlockManager::token_byte_size)
      .def_property_readonly("block_bytes", &BlockManager::block_bytes)
      .def_property_readonly("pool_bytes", &BlockManager::pool_bytes)
      .def("num_free", &BlockManager::num_free);

  py::class_<GraphWrapper>(m, "GraphWrapper", py::module_local())
      .def(py::init<>())
      .def("begin_capture",
           [](GraphWrapper& g, py::object s, int batch_size, int seq_len) { g.begin_capture(stream_of(s), batch_size, seq_len); },
           "Begin capturing operations into a graph on the given stream", py::arg("stream_obj"), py::arg("batch_size"),
           py::arg("seq_len"))
      .def("end_capture", [](GraphWrapper& g, py::object s) { g.end_capture(stream_of(s)); },
           "End graph capture and instantiate", py::arg("stream_obj"))
      .def("launch", &GraphWrapper::launch, "Replay the instantiated graph on each stream, holding buffer references",
           py::arg("stream_objs"), py::arg("buffers") = std::vector<py::object>())
      .def("is_valid", &GraphWrapper::is_valid, py::arg("batch_size"), py::arg("seq_len"))
      .def("invalidate", &GraphWrapper::invalidate)
      .def("block_table", &GraphWrapper::block_table)
      .def("in_flight", &GraphWrapper::in_flight)
      .def("pool_ptr", [](GraphWrapper& g) { return reinterpret_cast<uintptr_t>(g.block_manager().get_pool_ptr()); })
      .def("block_manager", &GraphWrapper::block_manager, py::return_value_policy::reference_internal);

  py::register_local_exception<HardwareMismatchError>(m, "HardwareMismatchError");

  auto desc = py::class_<KernelLaunchDescriptor>(m, "KernelLaunchDescriptor", py::module_local()).def(py::init<>());
#define KRT_FIELD(f) desc.def_readwrite(#f, &KernelLaunchDescriptor::f)
  KRT_FIELD(input_ptr); KRT_FIELD(output_ptr); KRT_FIELD(qkv_weight_ptr); KRT_FIELD(qkv_bias_ptr);
  KRT_FIELD(rms_weight_ptr); KRT_FIELD(freqs_cos_ptr); KRT_FIELD(freqs_sin_ptr); KRT_FIELD(k_output_ptr);
  KRT_FIELD(v_output_ptr); KRT_FIELD(seq_len); KRT_FIELD(d_model); KRT_FIELD(n_heads); KRT_FIELD(head_dim);
  KRT_FIELD(eps); KRT_FIELD(stride_x_seq); KRT_FIELD(stride_x_dim); KRT_FIELD(stride_w_out); KRT_FIELD(stride_w_in);
  KRT_FIELD(stride_q_seq); KRT_FIELD(stride_q_dim); KRT_FIELD(stride_k_seq); KRT_FIELD(stride_k_dim);
  KRT_FIELD(stride_v_seq); KRT_FIELD(stride_v_dim); KRT_FIELD(byte_size); KRT_FIELD(kernel_name); KRT_FIELD(grid_x);
  KRT_FIELD(grid_y); KRT_FIELD(grid_z); KRT_FIELD(block_x); KRT_FIELD(block_y); KRT_FIELD(block_z);
  KRT_FIELD(shared_mem_bytes);
  KRT_FIELD(dtype); KRT_FIELD(n_kv_heads); KRT_FIELD(positions_ptr); KRT_FIELD(token_seq_ptr);
  KRT_FIELD(block_table_ptr); KRT_FIELD(kv_pool_ptr); KRT_FIELD(num_seqs); KRT_FIELD(block_table_stride);
  KRT_FIELD(num_blocks); KRT_FIELD(tokens_per_block); KRT_FIELD(max_position); KRT_FIELD(workspace_ptr);
  KRT_FIELD(workspace_bytes);
#undef KRT_FIELD

  py::class_<AOTEngine>(m, "AOTEngine", py::module_local())
      .def(py::init<>())
      .def("compile_ahead_of_time",
           [](AOTEngine& e, const std::string& path, py::object s, const std::string& target) {
             e.compile_ahead_of_time(path, stream_of(s), target);
           },
           "Write a .kin artifact carrying the sm_100a kernel image", py::arg("output_filepath"),
           py::arg("stream_obj"), py::arg("kinetic_target"))
      .def("load_model", &AOTEngine::load_model, py::arg("filepath"))
      .def("launch",
           [](AOTEngine& e, const TensorDescriptor& in, const TensorDescriptor& out, int seq_len, py::object s) {
             validate_descriptor(in, "AOTEngine.launch.input");
             validate_descriptor(out, "AOTEngine.launch.output");
             e.launch(reinterpret_cast<void*>(in.data_ptr), reinterpret_cast<void*>(out.data_ptr), seq_len,
                      stream_of(s), in.byte_size);
           },
           py::arg("input"), py::arg("output"), py::arg("seq_len"), py::arg("stream_obj") = py::int_(0))
      .def("launch_tensor",
           [](AOTEngine& e, py::object in, py::object out, int seq_len, py::object s) {
             TensorDescriptor a = descriptor_from_tensor(in, "AOTEngine.launch_tensor.input");
             TensorDescriptor b = descriptor_from_tensor(out, "AOTEngine.launch_tensor.output");
             e.launch(reinterpret_cast<void*>(a.data_ptr), reinterpret_cast<void*>(b.data_ptr), seq_len, stream_of(s),
                      a.byte_size);
           },
           py::arg("input"), py::arg("output"), py::arg("seq_len"), py::arg("stream_obj") = py::int_(0))
      .def("launch",
           [](AOTEngine& e, uintptr_t in, uintptr_t out, int seq_len, py::object s, size_t byte_size) {
             e.launch(reinterpret_cast<void*>(in), reinterpret_cast<void*>(out), seq_len, stream_of(s), byte_size);
           },
           py::arg("input_ptr"), py::arg("output_ptr"), py::arg("seq_len"), py::arg("stream_obj") = py::int_(0),
           py::arg("byte_size") = 0)
      .def("launch_descriptor",
           [](AOTEngine& e, const KernelLaunchDescriptor& d, py::object s) { e.launch(d, stream_of(s)); },
           py::arg("descriptor"), py::arg("stream_obj"))
      .def("synchronize_and_clear", [](AOTEngine& e, py::object s) { e.synchronize_and_clear(stream_of(s)); },
           py::arg("stream_obj"));

  py::class_<Serializer>(m, "Serializer", py::module_local())
      .def(py::init<>())
      .def("save_kin_file", &Serializer::save_kin_file, py::arg("filepath"), py::arg("device_id"),
           py::arg("kinetic_target"), py::arg("weights_hash"), py::arg("op_graph_data"), py::arg("kernel_binaries"))
      .def("load_kin_file", &Serializer::load_kin_file, py::arg("filepath"))
      .def("get_tensor_parallel_degree", &Serializer::get_tensor_parallel_degree, py::arg("filepath"))
      .def_property_readonly("device_id", &Serializer::get_device_id);

  py::class_<Communicator>(m, "Communicator", py::module_local())
      .def(py::init<int, int>(), py::arg("rank"), py::arg("world_size"))
      .def("all_reduce_async",
           [](Communicator& c, uintptr_t send, uintptr_t recv, size_t count, int datatype, int op, py::object s) {
             const uintptr_t sp = stream_of(s);
             py::gil_scoped_release release;
             c.all_reduce_async(reinterpret_cast<void*>(send), reinterpret_cast<void*>(recv), count, datatype, op, sp);
           },
           "Allreduce-sum of `count` elements", py::arg("sendbuff"), py::arg("recvbuff"), py::arg("count"),
           py::arg("datatype"), py::arg("op"), py::arg("stream_obj"))
      .def("ipc_handle", [](Communicator& c) { return py::bytes(c.ipc_handle()); })
      .def("open_peers",
           [](Communicator& c, std::vector<py::bytes> hs) {
             std::vector<std::string> v;
             for (auto& h : hs) v.push_back(std::string(h));
             c.open_peers(v);
           },
           py::arg("handles"))
      .def("rowparallel_gemm_ar",
           [](Communicator& c, uintptr_t x, uintptr_t w, uintptr_t y, int num_tokens, int k_local, int n_out,
              int x_stride, int y_stride, py::object s) {
             c.rowparallel_gemm_ar(x, w, y, num_tokens, k_local, n_out, x_stride, y_stride, stream_of(s));
           },
           py::arg("x"), py::arg("weight"), py::arg("y"), py::arg("num_tokens"), py::arg("k_local"), py::arg("n_out"),
           py::arg("x_stride") = 0, py::arg("y_stride") = 0, py::arg("stream_obj") = py::int_(0))
      .def("read_status", [](Communicator& c, py::object s) { return c.read_status(stream_of(s)); },
           py::arg("stream_obj") = py::int_(0))
      .def_property_readonly("rank", &Communicator::rank)
      .def_property_readonly("world_size", &Communicator::world_size);

  py::class_<HardwareRouter>(m, "HardwareRouter", py::module_local())
      .def(py::init<>())
      .def("load_model", &HardwareRouter::load_model, py::arg("filepath"))
      .def("launch",
           [](HardwareRouter& r, const TensorDescriptor& in, const TensorDescriptor& out, int seq_len, size_t byte_size) {
             validate_descriptor(in, "HardwareRouter.launch.input");
             validate_descriptor(out, "HardwareRouter.launch.output");
             r.launch(reinterpret_cast<void*>(in.data_ptr), reinterpret_cast<void*>(out.data_ptr), seq_len,
                      byte_size ? byte_size : in.byte_size);
           },
           py::arg("input"), py::arg("output"), py::arg("seq_len"), py::arg("byte_size") = 0)
      .def("launch_tensor",
           [](HardwareRouter& r, py::object in, py::object out, int seq_len, size_t byte_size) {
             TensorDescriptor a = descriptor_from_tensor(in, "HardwareRouter.launch_tensor.input");
             TensorDescriptor b = descriptor_from_tensor(out, "HardwareRouter.launch_tensor.output");
             r.launch(reinterpret_cast<void*>(a.data_ptr), reinterpret_cast<void*>(b.data_ptr), seq_len,
                      byte_size ? byte_size : a.byte_size);
           },
           py::arg("input"), py::arg("output"), py::arg("seq_len"), py::arg("byte_size") = 0)
      .def("launch",
           [](HardwareRouter& r, uintptr_t in, uintptr_t out, int seq_len, size_t byte_size) {
             r.launch(reinterpret_cast<void*>(in), reinterpret_cast<void*>(out), seq_len, byte_size);
           },
           py::arg("input_ptr"), py::arg("output_ptr"), py::arg("seq_len"), py::arg("byte_size") = 0)
      .def_property_readonly("backend", &HardwareRouter::backend);

  py::class_<InferenceQueue>(m, "InferenceQueue", py::module_local())
      .def(py::init<>())
      .def("submit",
           [](InferenceQueue& q, const TensorDescriptor& in, int max_tokens, const std::string& id) {
             validate_descriptor(in, "InferenceQueue.submit.input");
             q.submit(in.data_ptr, numel_of(in), max_tokens, id);
           },
           py::arg("input"), py::arg("max_tokens"), py::arg("request_id"))
      .def("submit_tensor",
           [](InferenceQueue& q, py::object in, int max_tokens, const std::string& id) {
             TensorDescriptor d = descriptor_from_tensor(in, "InferenceQueue.submit_tensor.input");
             q.submit(d.data_ptr, numel_of(d), max_tokens, id);
           },
           py::arg("input"), py::arg("max_tokens"), py::arg("request_id"))
      .def("submit",
           [](InferenceQueue& q, uintptr_t p, size_t n, int max_tokens, const std::string& id) {
             q.submit(p, n, max_tokens, id);
           },
           py::arg("input_ptr"), py::arg("input_len"), py::arg("max_tokens"), py::arg("request_id"))
      .def("poll", &InferenceQueue::poll);

  py::class_<InferenceWorker>(m, "InferenceWorker", py::module_local())
      .def(py::init<InferenceQueue&, HardwareRouter&>(), py::arg("queue"), py::arg("router"), py::keep_alive<1, 2>(),
           py::keep_alive<1, 3>());

  // ---- per-request lifecycle (RequestContext.h)
  py::enum_<RequestState>(m, "RequestState", py::module_local())
      .value("RECEIVED", RequestState::RECEIVED).value("VALIDATED", RequestState::VALIDATED)
      .value("TOKENIZED", RequestState::TOKENIZED).value("ENQUEUED", RequestState::ENQUEUED)
      .value("PREFILL", RequestState::PREFILL).value("DECODE", RequestState::DECODE)
      .value("STREAMING", RequestState::STREAMING).value("COMPLETE", RequestState::COMPLETE)
      .value("CANCELLED", RequestState::CANCELLED).value("TIMED_OUT", RequestState::TIMED_OUT)
      .value("FAILED", RequestState::FAILED);
  py::enum_<CompletionReason>(m, "CompletionReason", py::module_local())
      .value("STREAMING", CompletionReason::STREAMING).value("EOS", CompletionReason::EOS)
      .value("STOP_TOKEN", CompletionReason::STOP_TOKEN).value("LENGTH", CompletionReason::LENGTH)
      .value("CANCELLED", CompletionReason::CANCELLED).value("TIMEOUT", CompletionReason::TIMEOUT)
      .value("ERROR", CompletionReason::ERROR);
  py::enum_<Owner>(m, "Owner", py::module_local())
      .value("Ingress", Owner::Ingress).value("Scheduler", Owner::Scheduler)
      .value("Executor", Owner::Executor).value("Backend", Owner::Backend);
  auto rc_error = py::register_local_exception<RequestContextError>(m, "RequestContextError", PyExc_RuntimeError);
  py::register_local_exception<InvalidStateTransitionError>(m, "InvalidStateTransitionError", rc_error);
  py::register_local_exception<RequestOwnershipError>(m, "RequestOwnershipError", rc_error);
  py::class_<RequestContext>(m, "RequestContext", py::module_local())
      .def(py::init([](std::string request_id, std::string prompt_text, std::vector<int32_t> prompt_tokens,
                       int max_new_tokens, float temperature, float top_p, int top_k,
                       std::vector<int32_t> stop_token_ids, std::string backend_hint, double timeout_s,
                       Owner initial_owner) {
             RequestContext::Config c;
             c.request_id = std::move(request_id);
             c.prompt_text = std::move(prompt_text);
             c.prompt_tokens = std::move(prompt_tokens);
             c.max_new_tokens = max_new_tokens;
             c.temperature = temperature;
             c.top_p = top_p;
             c.top_k = top_k;
             c.stop_token_ids = std::move(stop_token_ids);
             c.backend_hint = std::move(backend_hint);
             c.timeout = std::chrono::duration_cast<RequestContext::Clock::duration>(
                 std::chrono::duration<double>(timeout_s));
             c.initial_owner = initial_owner;
             return new RequestContext(std::move(c));
           }),
           py::arg("request_id"), py::arg("prompt_text") = "", py::arg("prompt_tokens") = std::vector<int32_t>{},
           py::arg("max_new_tokens") = 0, py::arg("temperature") = 1.0f, py::arg("top_p") = 1.0f,
           py::arg("top_k") = 0, py::arg("stop_token_ids") = std::vector<int32_t>{}, py::arg("backend_hint") = "",
           py::arg("timeout_s") = 0.0, py::arg("initial_owner") = Owner::Ingress)
      .def_property_readonly("request_id", &RequestContext::request_id)
      .def_property_readonly("prompt_text", &RequestContext::prompt_text)
      .def_property_readonly("prompt_tokens", &RequestContext::prompt_tokens)
      .def_property_readonly("max_new_tokens", &RequestContext::max_new_tokens)
      .def_property_readonly("stop_token_ids", &RequestContext::stop_token_ids)
      .def("is_valid", &RequestContext::is_valid)
      .def("ensure_executable", &RequestContext::ensure_executable)
      .def("state", &RequestContext::state)
      .def("can_transition_to", &RequestContext::can_transition_to)
      .def("transition_to", &RequestContext::transition_to)
      .def("is_terminal", py::overload_cast<>(&RequestContext::is_terminal, py::const_))
      .def("request_cancellation", &RequestContext::request_cancellation)
      .def("is_cancellation_requested", &RequestContext::is_cancellation_requested)
      .def("acknowledge_cancellation", &RequestContext::acknowledge_cancellation)
      .def("has_deadline", &RequestContext::has_deadline)
      .def("is_expired", [](const RequestContext& r) { return r.is_expired(); })
      .def("acknowledge_timeout", [](RequestContext& r) { r.acknowledge_timeout(); })
      .def("current_owner", &RequestContext::current_owner)
      .def("transfer_ownership", &RequestContext::transfer_ownership, py::arg("new_owner"),
           py::arg("expected_current_owner"))
      .def("append_generated_token", &RequestContext::append_generated_token)
      .def("generated_tokens", &RequestContext::generated_tokens)
      .def("set_kv_block_ids", &RequestContext::set_kv_block_ids)
      .def("kv_block_ids", &RequestContext::kv_block_ids)
      .def("set_finish_reason", &RequestContext::set_finish_reason)
      .def("finish_reason", &RequestContext::finish_reason)
      .def("set_error_code", &RequestContext::set_error_code)
      .def("error_code", &RequestContext::error_code)
      .def("register_cleanup_callback", &RequestContext::register_cleanup_callback)
      .def("is_cleaned_up", &RequestContext::is_cleaned_up)
      .def("cleanup", &RequestContext::cleanup);
}
