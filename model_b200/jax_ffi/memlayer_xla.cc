// XLA FFI handlers over the memory layer's C ABI: the binding that lets the
// reference's JAX / Flax code (memory_pool_model/memory.py:64-227 and the
// memory-layer block of model.py:108-120) call the sm_100a kernels as
// custom calls.  Built only where JAX is installed (its FFI headers come from
// jax.ffi.include_dir()); see model_b200/jax_ffi/__init__.py for the build,
// the registration and the Flax-facing functions.
//
// Every handler reads its shapes from the buffers and its MemoryPool
// fields from attributes, fills the C ABI structs and makes one call on the
// stream XLA gives it.  Scratch memory comes from XLA's scratch allocator;
// the library itself allocates nothing.
#include <cstdint>
#include <optional>
#include <string>

#include "memlayer.h"
#include "xla/ffi/api/ffi.h"

namespace ffi = xla::ffi;

namespace {

ffi::Error status_error(int32_t st, const char* where) {
  if (st == MEMLAYER_OK) return ffi::Error::Success();
  return ffi::Error(ffi::ErrorCode::kInternal, std::string(where) + ": " + memlayer_status_string(st));
}

int32_t dtype_of(ffi::DataType t) {
  switch (t) {
    case ffi::DataType::F16: return MEMLAYER_F16;
    case ffi::DataType::BF16: return MEMLAYER_BF16;
    default: return MEMLAYER_F32;
  }
}

memlayer_config config(int64_t tokens, int32_t heads, int32_t n_sub_keys, int32_t d_key, int32_t d_value,
                       int32_t top_k, int32_t d_model, ffi::DataType vdt, float routing_noise, float min_t,
                       float max_t, int32_t query_scale, int32_t btgrad) {
  memlayer_config c{};
  c.tokens = tokens;
  c.heads = heads;
  c.n_sub_keys = n_sub_keys;
  c.d_key = d_key;
  c.d_value = d_value;
  c.top_k = top_k;
  c.d_model = d_model;
  c.values_dtype = dtype_of(vdt);
  c.routing_noise = routing_noise;
  c.min_temperature = min_t;
  c.max_temperature = max_t;
  c.query_scale = query_scale;
  c.balance_temperature_grad = btgrad;
  return c;
}

template <class B>
const float* f32_or_null(const B& b) {
  return b.element_count() > 0 ? b.typed_data() : nullptr;
}

}  // namespace

// MemoryPool.__call__ (memory.py:119-227), inference or training with
// statistics.  gumbel: [M, H, 2, n] standard Gumbel sample, or an empty
// array when train == 0 (memory.py:155-159).
static ffi::Error PoolForward(cudaStream_t stream, ffi::ScratchAllocator scratch, ffi::Buffer<ffi::F32> queries,
                              ffi::Buffer<ffi::F32> sub_keys, ffi::Buffer<ffi::F32> log_t, ffi::AnyBuffer values,
                              ffi::Buffer<ffi::F32> gumbel, ffi::Result<ffi::Buffer<ffi::F32>> out,
                              ffi::Result<ffi::Buffer<ffi::S32>> slots, ffi::Result<ffi::Buffer<ffi::F32>> weights,
                              ffi::Result<ffi::Buffer<ffi::F32>> temperature,
                              ffi::Result<ffi::Buffer<ffi::F32>> top1_weight,
                              ffi::Result<ffi::Buffer<ffi::F32>> subkey_counts,
                              ffi::Result<ffi::Buffer<ffi::F32>> slot_counts,
                              ffi::Result<ffi::Buffer<ffi::F32>> balance_loss,
                              ffi::Result<ffi::Buffer<ffi::F32>> queries_unit, int32_t heads, int32_t n_sub_keys,
                              int32_t d_key, int32_t d_value, int32_t top_k, float routing_noise, float min_t,
                              float max_t, int32_t query_scale, int32_t btgrad, int32_t train, float noise_scale,
                              int32_t shuffle_reads, int32_t stats) {
  const int64_t M = queries.element_count() / ((int64_t)heads * d_key);
  const memlayer_config c = config(M, heads, n_sub_keys, d_key, d_value, top_k, 0, values.element_type(),
                                   routing_noise, min_t, max_t, query_scale, btgrad);
  memlayer_pool_args a{};
  a.queries = queries.typed_data();
  a.sub_keys = sub_keys.typed_data();
  a.log_temperature = log_t.typed_data();
  a.values = values.untyped_data();
  a.gumbel = f32_or_null(gumbel);
  a.noise_scale = noise_scale;
  a.train = train;
  a.shuffle_reads = shuffle_reads;
  a.out = out->typed_data();
  a.slots = slots->typed_data();
  a.weights = weights->typed_data();
  a.temperature = temperature->typed_data();
  a.top1_weight = top1_weight->typed_data();
  if (stats) {
    a.subkey_counts = subkey_counts->typed_data();
    a.slot_counts = slot_counts->typed_data();
    a.balance_loss = balance_loss->typed_data();
    a.queries_unit = queries_unit->typed_data();
  }
  size_t bytes = 0;
  int32_t st = memlayer_pool_workspace_size(&c, &bytes);
  if (st) return status_error(st, "memlayer_pool_workspace_size");
  std::optional<void*> ws = scratch.Allocate(bytes, 256);
  if (!ws) return ffi::Error(ffi::ErrorCode::kResourceExhausted, "memlayer: no scratch for the workspace");
  return status_error(memlayer_pool_forward(&c, &a, *ws, bytes, stream), "memlayer_pool_forward");
}

XLA_FFI_DEFINE_HANDLER_SYMBOL(MemlayerPoolForward, PoolForward,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Ctx<ffi::ScratchAllocator>()
                                  .Arg<ffi::Buffer<ffi::F32>>()    // queries [..., H, d_key]
                                  .Arg<ffi::Buffer<ffi::F32>>()    // sub_keys [H, 2, n, d_key / 2]
                                  .Arg<ffi::Buffer<ffi::F32>>()    // log_temperature [1]
                                  .Arg<ffi::AnyBuffer>()           // values [n * n, d] f32 / f16 / bf16
                                  .Arg<ffi::Buffer<ffi::F32>>()    // gumbel [M, H, 2, n] or [0]
                                  .Ret<ffi::Buffer<ffi::F32>>()    // out [M, d]
                                  .Ret<ffi::Buffer<ffi::S32>>()    // slots [M, H, k]
                                  .Ret<ffi::Buffer<ffi::F32>>()    // weights [M, H, k]
                                  .Ret<ffi::Buffer<ffi::F32>>()    // temperature [1]
                                  .Ret<ffi::Buffer<ffi::F32>>()    // top1_weight [1]
                                  .Ret<ffi::Buffer<ffi::F32>>()    // subkey_counts [H, 2, n] (stats)
                                  .Ret<ffi::Buffer<ffi::F32>>()    // slot_counts [n * n] (stats)
                                  .Ret<ffi::Buffer<ffi::F32>>()    // balance_loss [1] (stats)
                                  .Ret<ffi::Buffer<ffi::F32>>()    // queries_unit [M, H, 2, d_key / 2] (stats)
                                  .Attr<int32_t>("heads")
                                  .Attr<int32_t>("n_sub_keys")
                                  .Attr<int32_t>("d_key")
                                  .Attr<int32_t>("d_value")
                                  .Attr<int32_t>("top_k")
                                  .Attr<float>("routing_noise")
                                  .Attr<float>("min_temperature")
                                  .Attr<float>("max_temperature")
                                  .Attr<int32_t>("query_scale")
                                  .Attr<int32_t>("balance_temperature_grad")
                                  .Attr<int32_t>("train")
                                  .Attr<float>("noise_scale")
                                  .Attr<int32_t>("shuffle_reads")
                                  .Attr<int32_t>("stats"));

// The memory-layer block (model.py:110-119): y = Dense(mem * silu(Dense(h))),
// mem = MemoryPool(Dense(h)).  Returns the forward workspace as an output
// (`residual`, memlayer_layer_workspace_size bytes), which the backward's
// balance term reads unchanged.
static ffi::Error LayerForward(cudaStream_t stream, ffi::Buffer<ffi::F32> h, ffi::Buffer<ffi::F32> w_router,
                               ffi::Buffer<ffi::F32> b_router, ffi::Buffer<ffi::F32> w_gate,
                               ffi::Buffer<ffi::F32> b_gate, ffi::Buffer<ffi::F32> w_out, ffi::Buffer<ffi::F32> b_out,
                               ffi::Buffer<ffi::F32> sub_keys, ffi::Buffer<ffi::F32> log_t, ffi::AnyBuffer values,
                               ffi::Buffer<ffi::F32> gumbel, ffi::Result<ffi::Buffer<ffi::F32>> y,
                               ffi::Result<ffi::Buffer<ffi::F32>> mem, ffi::Result<ffi::Buffer<ffi::S32>> slots,
                               ffi::Result<ffi::Buffer<ffi::F32>> weights,
                               ffi::Result<ffi::Buffer<ffi::F32>> temperature,
                               ffi::Result<ffi::Buffer<ffi::F32>> top1_weight,
                               ffi::Result<ffi::Buffer<ffi::F32>> subkey_counts,
                               ffi::Result<ffi::Buffer<ffi::F32>> slot_counts,
                               ffi::Result<ffi::Buffer<ffi::F32>> balance_loss,
                               ffi::Result<ffi::Buffer<ffi::U8>> residual, int32_t heads, int32_t n_sub_keys,
                               int32_t d_key, int32_t d_value, int32_t top_k, int32_t d_model, float routing_noise,
                               float min_t, float max_t, int32_t query_scale, int32_t btgrad, int32_t train,
                               float noise_scale, int32_t shuffle_reads, int32_t stats) {
  const int64_t M = h.element_count() / d_model;
  const memlayer_config c = config(M, heads, n_sub_keys, d_key, d_value, top_k, d_model, values.element_type(),
                                   routing_noise, min_t, max_t, query_scale, btgrad);
  memlayer_layer_args a{};
  a.h = h.typed_data();
  a.w_router = w_router.typed_data();
  a.b_router = f32_or_null(b_router);
  a.w_gate = w_gate.typed_data();
  a.b_gate = f32_or_null(b_gate);
  a.w_out = w_out.typed_data();
  a.b_out = f32_or_null(b_out);
  a.y = y->typed_data();
  a.mem = mem->typed_data();
  a.pool.sub_keys = sub_keys.typed_data();
  a.pool.log_temperature = log_t.typed_data();
  a.pool.values = values.untyped_data();
  a.pool.gumbel = f32_or_null(gumbel);
  a.pool.noise_scale = noise_scale;
  a.pool.train = train;
  a.pool.shuffle_reads = shuffle_reads;
  a.pool.slots = slots->typed_data();
  a.pool.weights = weights->typed_data();
  a.pool.temperature = temperature->typed_data();
  a.pool.top1_weight = top1_weight->typed_data();
  if (stats) {
    a.pool.subkey_counts = subkey_counts->typed_data();
    a.pool.slot_counts = slot_counts->typed_data();
    a.pool.balance_loss = balance_loss->typed_data();
  }
  return status_error(memlayer_layer_forward(&c, &a, residual->untyped_data(), residual->size_bytes(), stream),
                      "memlayer_layer_forward");
}

XLA_FFI_DEFINE_HANDLER_SYMBOL(MemlayerLayerForward, LayerForward,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()    // h [M, d_model]
                                  .Arg<ffi::Buffer<ffi::F32>>()    // router_i kernel [d_model, H * d_key]
                                  .Arg<ffi::Buffer<ffi::F32>>()    // router_i bias (or [0])
                                  .Arg<ffi::Buffer<ffi::F32>>()    // mem_gate_i kernel [d_model, d]
                                  .Arg<ffi::Buffer<ffi::F32>>()    // mem_gate_i bias (or [0])
                                  .Arg<ffi::Buffer<ffi::F32>>()    // mem_out_i kernel [d, d_model]
                                  .Arg<ffi::Buffer<ffi::F32>>()    // mem_out_i bias (or [0])
                                  .Arg<ffi::Buffer<ffi::F32>>()    // sub_keys
                                  .Arg<ffi::Buffer<ffi::F32>>()    // log_temperature [1]
                                  .Arg<ffi::AnyBuffer>()           // values
                                  .Arg<ffi::Buffer<ffi::F32>>()    // gumbel or [0]
                                  .Ret<ffi::Buffer<ffi::F32>>()    // y [M, d_model]
                                  .Ret<ffi::Buffer<ffi::F32>>()    // mem [M, d]
                                  .Ret<ffi::Buffer<ffi::S32>>()    // slots
                                  .Ret<ffi::Buffer<ffi::F32>>()    // weights
                                  .Ret<ffi::Buffer<ffi::F32>>()    // temperature [1]
                                  .Ret<ffi::Buffer<ffi::F32>>()    // top1_weight [1]
                                  .Ret<ffi::Buffer<ffi::F32>>()    // subkey_counts (stats)
                                  .Ret<ffi::Buffer<ffi::F32>>()    // slot_counts (stats)
                                  .Ret<ffi::Buffer<ffi::F32>>()    // balance_loss (stats)
                                  .Ret<ffi::Buffer<ffi::U8>>()     // residual: the forward workspace
                                  .Attr<int32_t>("heads")
                                  .Attr<int32_t>("n_sub_keys")
                                  .Attr<int32_t>("d_key")
                                  .Attr<int32_t>("d_value")
                                  .Attr<int32_t>("top_k")
                                  .Attr<int32_t>("d_model")
                                  .Attr<float>("routing_noise")
                                  .Attr<float>("min_temperature")
                                  .Attr<float>("max_temperature")
                                  .Attr<int32_t>("query_scale")
                                  .Attr<int32_t>("balance_temperature_grad")
                                  .Attr<int32_t>("train")
                                  .Attr<float>("noise_scale")
                                  .Attr<int32_t>("shuffle_reads")
                                  .Attr<int32_t>("stats"));

// Gradients of sum(dy * y) + balance_coef * balance_loss through the block
// (the reference trainer's value_and_grad with sparse_grad, train.py:305-335):
// the Dense, sub-key and temperature gradients, d h, and the read-output
// gradient `probe` that feeds the fetched-row update.
static ffi::Error LayerBackward(cudaStream_t stream, ffi::ScratchAllocator scratch, ffi::Buffer<ffi::F32> h,
                                ffi::Buffer<ffi::F32> w_router, ffi::Buffer<ffi::F32> b_router,
                                ffi::Buffer<ffi::F32> w_gate, ffi::Buffer<ffi::F32> b_gate,
                                ffi::Buffer<ffi::F32> w_out, ffi::Buffer<ffi::F32> b_out,
                                ffi::Buffer<ffi::F32> sub_keys, ffi::Buffer<ffi::F32> log_t, ffi::AnyBuffer values,
                                ffi::Buffer<ffi::S32> slots, ffi::Buffer<ffi::F32> weights,
                                ffi::Buffer<ffi::F32> balance_loss, ffi::Buffer<ffi::U8> residual,
                                ffi::Buffer<ffi::F32> dy, ffi::Result<ffi::Buffer<ffi::F32>> dh,
                                ffi::Result<ffi::Buffer<ffi::F32>> dw_router,
                                ffi::Result<ffi::Buffer<ffi::F32>> db_router,
                                ffi::Result<ffi::Buffer<ffi::F32>> dsub_keys,
                                ffi::Result<ffi::Buffer<ffi::F32>> dlog_t, ffi::Result<ffi::Buffer<ffi::F32>> dw_gate,
                                ffi::Result<ffi::Buffer<ffi::F32>> db_gate, ffi::Result<ffi::Buffer<ffi::F32>> dw_out,
                                ffi::Result<ffi::Buffer<ffi::F32>> db_out, ffi::Result<ffi::Buffer<ffi::F32>> probe,
                                int32_t heads, int32_t n_sub_keys, int32_t d_key, int32_t d_value, int32_t top_k,
                                int32_t d_model, float routing_noise, float min_t, float max_t, int32_t query_scale,
                                int32_t btgrad, int32_t shuffle_reads, float balance_coef,
                                int32_t route_through_pool) {
  const int64_t M = h.element_count() / d_model;
  const memlayer_config c = config(M, heads, n_sub_keys, d_key, d_value, top_k, d_model, values.element_type(),
                                   routing_noise, min_t, max_t, query_scale, btgrad);
  memlayer_layer_args a{};
  a.h = h.typed_data();
  a.w_router = w_router.typed_data();
  a.b_router = f32_or_null(b_router);
  a.w_gate = w_gate.typed_data();
  a.b_gate = f32_or_null(b_gate);
  a.w_out = w_out.typed_data();
  a.b_out = f32_or_null(b_out);
  a.pool.sub_keys = sub_keys.typed_data();
  a.pool.log_temperature = log_t.typed_data();
  a.pool.values = values.untyped_data();
  a.pool.shuffle_reads = shuffle_reads;
  a.pool.slots = const_cast<int32_t*>(slots.typed_data());
  a.pool.weights = const_cast<float*>(weights.typed_data());
  a.pool.balance_loss = const_cast<float*>(f32_or_null(balance_loss));
  memlayer_layer_grads g{};
  g.dy = dy.typed_data();
  g.balance_coef = balance_coef;
  g.route_through_pool = route_through_pool;
  g.forward_workspace = residual.untyped_data();
  g.dh = dh->typed_data();
  g.dw_router = dw_router->typed_data();
  g.db_router = db_router->typed_data();
  g.dsub_keys = dsub_keys->typed_data();
  g.dlog_temperature = dlog_t->typed_data();
  g.dw_gate = dw_gate->typed_data();
  g.db_gate = db_gate->typed_data();
  g.dw_out = dw_out->typed_data();
  g.db_out = db_out->typed_data();
  g.probe = probe->typed_data();
  size_t bytes = 0;
  int32_t st = memlayer_layer_backward_workspace_size(&c, balance_coef != 0.f, &bytes);
  if (st) return status_error(st, "memlayer_layer_backward_workspace_size");
  std::optional<void*> ws = scratch.Allocate(bytes, 256);
  if (!ws) return ffi::Error(ffi::ErrorCode::kResourceExhausted, "memlayer: no scratch for the workspace");
  return status_error(memlayer_layer_backward(&c, &a, &g, *ws, bytes, stream), "memlayer_layer_backward");
}

XLA_FFI_DEFINE_HANDLER_SYMBOL(MemlayerLayerBackward, LayerBackward,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Ctx<ffi::ScratchAllocator>()
                                  .Arg<ffi::Buffer<ffi::F32>>()    // h
                                  .Arg<ffi::Buffer<ffi::F32>>()    // router kernel
                                  .Arg<ffi::Buffer<ffi::F32>>()    // router bias (or [0])
                                  .Arg<ffi::Buffer<ffi::F32>>()    // gate kernel
                                  .Arg<ffi::Buffer<ffi::F32>>()    // gate bias (or [0])
                                  .Arg<ffi::Buffer<ffi::F32>>()    // out kernel
                                  .Arg<ffi::Buffer<ffi::F32>>()    // out bias (or [0])
                                  .Arg<ffi::Buffer<ffi::F32>>()    // sub_keys
                                  .Arg<ffi::Buffer<ffi::F32>>()    // log_temperature
                                  .Arg<ffi::AnyBuffer>()           // values
                                  .Arg<ffi::Buffer<ffi::S32>>()    // the forward's slots
                                  .Arg<ffi::Buffer<ffi::F32>>()    // the forward's weights
                                  .Arg<ffi::Buffer<ffi::F32>>()    // the forward's balance_loss (or [0])
                                  .Arg<ffi::Buffer<ffi::U8>>()     // the forward's residual workspace
                                  .Arg<ffi::Buffer<ffi::F32>>()    // dy [M, d_model]
                                  .Ret<ffi::Buffer<ffi::F32>>()    // dh
                                  .Ret<ffi::Buffer<ffi::F32>>()    // d router kernel
                                  .Ret<ffi::Buffer<ffi::F32>>()    // d router bias
                                  .Ret<ffi::Buffer<ffi::F32>>()    // d sub_keys
                                  .Ret<ffi::Buffer<ffi::F32>>()    // d log_temperature
                                  .Ret<ffi::Buffer<ffi::F32>>()    // d gate kernel
                                  .Ret<ffi::Buffer<ffi::F32>>()    // d gate bias
                                  .Ret<ffi::Buffer<ffi::F32>>()    // d out kernel
                                  .Ret<ffi::Buffer<ffi::F32>>()    // d out bias
                                  .Ret<ffi::Buffer<ffi::F32>>()    // probe [M, d]
                                  .Attr<int32_t>("heads")
                                  .Attr<int32_t>("n_sub_keys")
                                  .Attr<int32_t>("d_key")
                                  .Attr<int32_t>("d_value")
                                  .Attr<int32_t>("top_k")
                                  .Attr<int32_t>("d_model")
                                  .Attr<float>("routing_noise")
                                  .Attr<float>("min_temperature")
                                  .Attr<float>("max_temperature")
                                  .Attr<int32_t>("query_scale")
                                  .Attr<int32_t>("balance_temperature_grad")
                                  .Attr<int32_t>("shuffle_reads")
                                  .Attr<float>("balance_coef")
                                  .Attr<int32_t>("route_through_pool"));
