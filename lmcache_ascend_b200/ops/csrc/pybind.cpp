// N1: the extension module.  Op names follow the reference's pybind module
// (csrc/pybind.cpp:243-483) where the op exists there; the layout objects
// (PagedLayout, ChunkLayout) are this framework's own descriptors.
#include <torch/extension.h>

#include <tuple>

#include "mem_kernels.h"

namespace lmc {
// mem_alloc.cpp
int64_t alloc_pinned_ptr(int64_t size, int64_t device);
void free_pinned_ptr(int64_t ptr);
int64_t alloc_pinned_numa_ptr(int64_t size, int64_t numa_node);
void free_pinned_numa_ptr(int64_t ptr);
int64_t alloc_shm_pinned_ptr(int64_t size, const std::string &name, int64_t numa_node);
int64_t attach_shm_pinned_ptr(int64_t size, const std::string &name);
void detach_shm_pinned_ptr(int64_t ptr);
void free_shm_pinned_ptr(int64_t ptr);
void unlink_shm(const std::string &name);
int64_t register_mapping(int64_t ptr, int64_t size);
void unregister_ptr(int64_t ptr);
int64_t get_device_ptr(int64_t ptr);
at::Tensor host_tensor_view(int64_t ptr, int64_t size);
int64_t registered_bytes();
// ipc.cpp
std::tuple<pybind11::bytes, int64_t, int64_t> ipc_export(int64_t ptr, int64_t device);
int64_t ipc_import(const std::string &handle, int64_t offset, int64_t device);
void ipc_close(const std::string &handle);
int64_t ipc_open_count();
at::Tensor device_buffer(int64_t nbytes, int64_t device);
bool enable_peer_access(int64_t device, int64_t peer);
std::string get_gpu_pci_bus_id(int64_t device);
// pd_push.cu
int64_t push_units_per_layer(int64_t num_tokens, int64_t num_planes, int64_t tile_tokens);
void pd_push(const PagedLayout &src, const PagedLayout &dst, const at::Tensor &src_slots,
             const at::Tensor &dst_slots, int64_t layer_begin, int64_t num_layers,
             int64_t replicas, const std::vector<int64_t> &flag_ptrs, int64_t tile_tokens,
             int64_t grid, const c10::optional<at::Tensor> &status, int64_t mode,
             const c10::optional<at::Tensor> &counters, bool local_dst);
int64_t fp8_staging_bytes(const PagedLayout &layout, int64_t num_tokens, int64_t num_layers,
                          int64_t group, bool scales);
void pd_push_fp8(const PagedLayout &src, int64_t q_ptr, int64_t scale_ptr,
                 const at::Tensor &src_slots, int64_t layer_begin, int64_t num_layers,
                 int64_t flag_ptr, int64_t tile_tokens, int64_t grid, int64_t group,
                 const c10::optional<at::Tensor> &status, bool local_dst);
void pd_dequant_scatter(const PagedLayout &dst, int64_t q_ptr, int64_t scale_ptr,
                        const at::Tensor &dst_slots, int64_t layer_begin, int64_t num_layers,
                        int64_t group, const c10::optional<at::Tensor> &status);
void pd_push_multimem(const PagedLayout &src, int64_t mc_rows, int64_t mc_flags,
                      const at::Tensor &src_slots, int64_t layer_begin, int64_t num_layers,
                      int64_t tile_tokens, int64_t grid,
                      const c10::optional<at::Tensor> &status);
void pd_wait_value(int64_t flag_ptr, int64_t target, double timeout_s,
                   const c10::optional<at::Tensor> &status);
void pd_flag_add(int64_t flag_ptr, int64_t inc);
void pd_wait_flags(int64_t flags_ptr, const at::Tensor &targets, int64_t layer_begin,
                   double timeout_s, const c10::optional<at::Tensor> &status);
// cachegen_kernels.cu
at::Tensor cachegen_cdf_from_lengths(const at::Tensor &packed, int64_t rows, int64_t channels,
                                     int64_t bins);
void c8_copy(const at::Tensor &planes, const at::Tensor &slots, const at::Tensor &packets,
             int64_t cap, int64_t num_layers, int64_t key_bytes, int64_t factor,
             const c10::optional<at::Tensor> &block_map, int64_t cache_slots,
             int64_t phys_limit, bool to_packet);
void cachegen_compact(const at::Tensor &src, const at::Tensor &cap, const at::Tensor &first,
                      const at::Tensor &lengths, const at::Tensor &offsets, at::Tensor &dst);
at::Tensor calculate_cdf(const at::Tensor &input, int64_t n_bins);
void encode_fast_new(const at::Tensor &cdf, const at::Tensor &input_sym,
                     at::Tensor &output_buffer, at::Tensor &output_lengths,
                     const c10::optional<at::Tensor> &status);
void decode_fast_prefsum(const at::Tensor &cdf, const at::Tensor &bytestreams,
                         const at::Tensor &lengths, at::Tensor &output);
// pos_kernels.cu
void cachegen_quantize(const at::Tensor &x, const at::Tensor &bins, at::Tensor &sym,
                       at::Tensor &scale, const c10::optional<at::Tensor> &row_dst);
void cachegen_dequantize(const at::Tensor &sym, const at::Tensor &scale, const at::Tensor &bins,
                         at::Tensor &y, const c10::optional<at::Tensor> &row_src);
void rotary_embedding_k_fused(const at::Tensor &old_positions, const at::Tensor &new_positions,
                              at::Tensor &key, int64_t head_size,
                              const at::Tensor &cos_sin_cache, bool is_neox,
                              const c10::optional<at::Tensor> &slot_mapping);
void rotary_embedding_k_fused_layers(const at::Tensor &old_positions,
                                     const at::Tensor &new_positions,
                                     const std::vector<at::Tensor> &keys, int64_t head_size,
                                     const at::Tensor &cos_sin_cache, bool is_neox,
                                     const c10::optional<at::Tensor> &slot_mapping);
// dma.cu
void dma_copy_batch(const at::Tensor &dsts, const at::Tensor &srcs, const at::Tensor &sizes);
double dma_copy_batch_timed(const at::Tensor &dsts, const at::Tensor &srcs,
                            const at::Tensor &sizes);
void gather_copy(const at::Tensor &table);
}  // namespace lmc

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  using namespace lmc;
  namespace py = pybind11;
  m.doc() = "lmcache_ascend_b200 native ops (sm_100a)";

  py::class_<PagedLayout>(m, "PagedLayout")
      .def(py::init<at::Tensor, std::vector<int64_t>, std::vector<int64_t>,
                    std::vector<int64_t>, int64_t, int64_t, std::vector<int64_t>,
                    std::vector<int64_t>>(),
           py::arg("ptrs"), py::arg("block_stride"), py::arg("slot_stride"),
           py::arg("row_bytes"), py::arg("block_size"), py::arg("num_slots"),
           py::arg("seg_bytes") = std::vector<int64_t>{},
           py::arg("seg_stride") = std::vector<int64_t>{})
      .def_property_readonly("segmented", &PagedLayout::segmented)
      .def("set_bases_aligned", &PagedLayout::set_bases_aligned)
      .def_property_readonly("aligned", &PagedLayout::aligned)
      .def_property_readonly("num_layers", &PagedLayout::num_layers)
      .def_property_readonly("num_planes", &PagedLayout::num_planes)
      .def_property_readonly("ptrs", &PagedLayout::ptrs);

  py::class_<ChunkLayout>(m, "ChunkLayout")
      .def(py::init<std::vector<int64_t>, int64_t, std::vector<int64_t>,
                    std::vector<int64_t>>(),
           py::arg("plane_stride_t"), py::arg("layer_stride_t"),
           py::arg("token_stride"), py::arg("col_off"));

  m.def("kv_transfer", &kv_transfer, py::arg("paged"), py::arg("chunk"),
        py::arg("chunk_ptrs"), py::arg("layout"), py::arg("chunk_ntok"),
        py::arg("chunk_tok_off"), py::arg("chunk_tokens"), py::arg("chunk_on_device"),
        py::arg("slots"), py::arg("layer_begin"), py::arg("chunk_layer_begin"),
        py::arg("num_layers"), py::arg("to_chunk"), py::arg("mode") = 0,
        py::arg("status") = py::none(), py::arg("chunk_idx") = py::none(),
        py::arg("chunk_idx_limit") = 0, py::arg("num_tokens_dev") = py::none(),
        "paged <-> chunk transfer (TMA bulk or SIMT engine)");
  m.def("num_sms", &num_sms);
  m.def("fused_multi_layer_kv_transfer", &fused_multi_layer_kv_transfer,
        py::arg("host_chunk"), py::arg("staging"), py::arg("paged"), py::arg("layout"),
        py::arg("slots"), py::arg("from_gpu"), py::arg("mode") = 0,
        py::arg("status") = py::none(),
        "paged <-> pinned host chunk through a device staging buffer");
  m.def("paged_copy", &paged_copy, py::arg("src"), py::arg("dst"), py::arg("src_slots"),
        py::arg("dst_slots"), py::arg("layer_begin"), py::arg("dst_layer_begin"),
        py::arg("num_layers"), py::arg("mode") = 0, py::arg("status") = py::none(),
        py::arg("flags_ptr") = 0, py::arg("flag_inc") = 0,
        "paged -> paged copy on one GPU (TMA bulk or SIMT), optional flag release");

  m.def("alloc_pinned_ptr", &alloc_pinned_ptr, py::arg("size"), py::arg("device") = -1);
  m.def("free_pinned_ptr", &free_pinned_ptr);
  m.def("alloc_pinned_numa_ptr", &alloc_pinned_numa_ptr);
  m.def("free_pinned_numa_ptr", &free_pinned_numa_ptr);
  m.def("alloc_shm_pinned_ptr", &alloc_shm_pinned_ptr, py::arg("size"), py::arg("name"),
        py::arg("numa_node") = -1);
  m.def("attach_shm_pinned_ptr", &attach_shm_pinned_ptr);
  m.def("detach_shm_pinned_ptr", &detach_shm_pinned_ptr);
  m.def("free_shm_pinned_ptr", &free_shm_pinned_ptr);
  m.def("unlink_shm", &unlink_shm);
  m.def("register_mapping", &register_mapping);
  m.def("unregister_ptr", &unregister_ptr);
  m.def("get_device_ptr", &get_device_ptr);
  m.def("host_tensor_view", &host_tensor_view);
  m.def("registered_bytes", &registered_bytes);

  m.def("ipc_export", &ipc_export, py::arg("ptr"), py::arg("device"));
  m.def("ipc_import", [](py::bytes h, int64_t off, int64_t dev) {
    return ipc_import(std::string(h), off, dev);
  });
  m.def("ipc_close", [](py::bytes h) { ipc_close(std::string(h)); });
  m.def("ipc_open_count", &ipc_open_count);
  m.def("device_buffer", &device_buffer);
  m.def("enable_peer_access", &enable_peer_access);
  m.def("get_gpu_pci_bus_id", &get_gpu_pci_bus_id);

  m.def("push_units_per_layer", &push_units_per_layer);
  m.def("pd_push", &pd_push, py::arg("src"), py::arg("dst"), py::arg("src_slots"),
        py::arg("dst_slots"), py::arg("layer_begin"), py::arg("num_layers"),
        py::arg("replicas") = 1, py::arg("flag_ptrs") = std::vector<int64_t>{},
        py::arg("tile_tokens") = 128, py::arg("grid") = 0,
        py::arg("status") = py::none(), py::arg("mode") = 0,
        py::arg("counters") = py::none(), py::arg("local_dst") = false);
  m.def("fp8_staging_bytes", &fp8_staging_bytes);
  m.def("pd_push_multimem", &pd_push_multimem, py::arg("src"), py::arg("mc_rows"),
        py::arg("mc_flags"), py::arg("src_slots"), py::arg("layer_begin"),
        py::arg("num_layers"), py::arg("tile_tokens") = 128, py::arg("grid") = 0,
        py::arg("status") = py::none());
  m.def("pd_push_fp8", &pd_push_fp8, py::arg("src"), py::arg("q_ptr"), py::arg("scale_ptr"),
        py::arg("src_slots"), py::arg("layer_begin"), py::arg("num_layers"),
        py::arg("flag_ptr"), py::arg("tile_tokens") = 128, py::arg("grid") = 0,
        py::arg("group") = 128, py::arg("status") = py::none(),
        py::arg("local_dst") = false);
  m.def("pd_dequant_scatter", &pd_dequant_scatter, py::arg("dst"), py::arg("q_ptr"),
        py::arg("scale_ptr"), py::arg("dst_slots"), py::arg("layer_begin"),
        py::arg("num_layers"), py::arg("group") = 128, py::arg("status") = py::none());
  m.def("pd_wait_flags", &pd_wait_flags, py::arg("flags_ptr"), py::arg("targets"),
        py::arg("layer_begin"), py::arg("timeout_s"), py::arg("status") = py::none());
  m.def("pd_wait_value", &pd_wait_value, py::arg("flag_ptr"), py::arg("target"),
        py::arg("timeout_s"), py::arg("status") = py::none());
  m.def("pd_flag_add", &pd_flag_add, py::arg("flag_ptr"), py::arg("inc") = 1);

  m.def("calculate_cdf", &calculate_cdf);
  m.def("encode_fast_new", &encode_fast_new, py::arg("cdf"), py::arg("input_sym"),
        py::arg("output_buffer"), py::arg("output_lengths"),
        py::arg("status") = py::none());
  m.def("decode_fast_prefsum", &decode_fast_prefsum);
  m.def("cachegen_cdf_from_lengths", &cachegen_cdf_from_lengths);
  m.def("c8_copy", &c8_copy);
  m.def("cachegen_compact", &cachegen_compact);
  m.def("cachegen_quantize", &cachegen_quantize, py::arg("x"), py::arg("bins"), py::arg("sym"),
        py::arg("scale"), py::arg("row_dst") = py::none());
  m.def("cachegen_dequantize", &cachegen_dequantize, py::arg("sym"), py::arg("scale"),
        py::arg("bins"), py::arg("y"), py::arg("row_src") = py::none());
  m.def("rotary_embedding_k_fused_layers", &rotary_embedding_k_fused_layers,
        py::arg("old_positions"), py::arg("new_positions"), py::arg("keys"),
        py::arg("head_size"), py::arg("cos_sin_cache"), py::arg("is_neox"),
        py::arg("slot_mapping") = py::none());
  m.def("rotary_embedding_k_fused", &rotary_embedding_k_fused, py::arg("old_positions"),
        py::arg("new_positions"), py::arg("key"), py::arg("head_size"),
        py::arg("cos_sin_cache"), py::arg("is_neox"), py::arg("slot_mapping") = py::none());

  m.def("layerwise_prefill_dma_copy", &dma_copy_batch);
  m.def("layerwise_prefill_dma_copy_diagnose", &dma_copy_batch_timed);
  m.def("gather_copy", &gather_copy);
}
