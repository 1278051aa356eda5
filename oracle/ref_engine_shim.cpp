// C shim over the reference's compiled-model catalog engine
// (native/src/engine/model_engine_compiled.cpp, compiled unmodified next to
// this file into oracle/_ref/libref_engine.so). It lets a test load a
// models.tsv catalog of this repository's model libraries exactly the way
// the reference's workers do: Engine (catalog parse, dlopen, dlsym of the
// seven ABI symbols, PpocrModelInfo validation, shared weights per file),
// then Context::select_profile / set_input_shape / bind_workspace / enqueue
// (model_engine_compiled.cpp:76-156).
// TEST INFRASTRUCTURE ONLY.
#include "ppocrv6_native/engine/model_engine.h"
#include <cstring>
#include <memory>
#include <string>

using namespace ppocrv6_native::engine;

namespace {
thread_local std::string g_error;
struct Handle {
  std::unique_ptr<ModelEngine> engine;
  std::unique_ptr<ModelContext> context;
};
} // namespace

extern "C" {

const char *ref_engine_error(void) { return g_error.c_str(); }

void *ref_engine_load(const char *catalog) {
  try {
    auto h = std::make_unique<Handle>();
    h->engine = load_model_engine(catalog);
    h->context = h->engine->create_context();
    return h.release();
  } catch (const std::exception &e) {
    g_error = e.what();
    return nullptr;
  }
}

int ref_engine_profiles(void *handle) {
  return static_cast<Handle *>(handle)->engine->profiles();
}

// Input shape of a profile at its maximum batch: out[0..3].
void ref_engine_profile_shape(void *handle, int profile, long long *out) {
  const TensorShape s = static_cast<Handle *>(handle)->engine->profile_shape(profile, true);
  for (int i = 0; i < 4; ++i)
    out[i] = s.d[i];
}

long long ref_engine_workspace_bytes(void *handle) {
  return static_cast<Handle *>(handle)->engine->workspace_bytes(-1);
}

int ref_engine_output_is_f32(void *handle) {
  return static_cast<Handle *>(handle)->engine->output_type() == ElementType::Float32;
}

// One inference: profile, batch x (C,H,W of the profile) f32 NCHW input on
// the device, output on the device, the caller's scratch of
// ref_engine_workspace_bytes bytes.
int ref_engine_enqueue(void *handle, int profile, int batch, const float *input, void *output,
                       void *scratch, long long scratch_bytes, cudaStream_t stream) {
  try {
    auto *h = static_cast<Handle *>(handle);
    if (!h->context->select_profile(profile, stream))
      throw std::runtime_error("select_profile rejected");
    const TensorShape m = h->engine->profile_shape(profile, true);
    if (!h->context->set_input_shape({batch, m.d[1], m.d[2], m.d[3]}))
      throw std::runtime_error("set_input_shape rejected");
    h->context->bind_workspace(scratch, scratch_bytes);
    h->context->enqueue(input, output, stream);
    return 0;
  } catch (const std::exception &e) {
    g_error = e.what();
    return -1;
  }
}

void ref_engine_destroy(void *handle) { delete static_cast<Handle *>(handle); }

} // extern "C"
