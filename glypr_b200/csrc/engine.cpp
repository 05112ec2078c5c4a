// Dynamic-batching inference engine: the production caller of the embedding path, after
// glypr-server's engine (crates/glypr-server/src/engine.rs:157-325).
//
// Any number of client threads call glp_engine_embed (blocking, like EngineHandle::embed
// awaiting its oneshot reply, engine.rs:120-150); requests wait in a bounded queue (1024 in
// the reference, mpsc::channel(1024)); one worker thread forms batches exactly as the
// reference's worker does — block for the first request, drain whatever is pending up to
// max_batch, yield once to let concurrently arriving requests in, drain again (engine.rs:
// 216-245) — and runs each batch through one executor call: glp_embed_tokens on the model
// context (which shards the batch across the context's devices), or a caller-supplied batch
// function.  Every request of a batch gets its full-width row, Matryoshka-truncated on the
// host when it asked for fewer dimensions (truncate_mrl, util.rs:6-29, as process_batch
// does, engine.rs:300-306); when the batch fails every request gets the error ("Batch inference error: ...", engine.rs:311-318).  Sequences need no length
// bucketing: the executor packs valid tokens, so batching requests of mixed lengths computes
// no padding.
//
// Destroying the engine lets the worker finish every queued request, then joins it; calls
// made after that are rejected ("Inference worker is not running", engine.rs:146-148).
#include <algorithm>
#include <cmath>
#include <condition_variable>
#include <cstring>
#include <exception>
#include <deque>
#include <mutex>
#include <string>
#include <string_view>
#include <thread>
#include <vector>

#include "glypr_cuda.h"

namespace glp {
void set_last_error(const std::string& msg);  // glypr_cuda.cu: this thread's glp_last_error()
// tokenizer.cpp
std::string tokenize_text(const glp_tokenizer* tok, std::string_view text, int form, std::vector<int32_t>* ids);
std::string format_task(const char* task, const char* title, std::string_view text);
bool valid_utf8(const char* s, size_t n);
}

namespace {

struct Request {
  const int32_t* ids = nullptr;
  int len = 0;
  int truncate_dim = 0;  // 0 or >= the embedding width: full width
  float* out = nullptr;
  int rc = GLP_OK;
  std::string err;
  bool done = false;
};

int model_batch(void* user, const int32_t* ids, const int32_t* lengths, int n_seq, int max_len, int out_dim,
                float* out) {
  return glp_embed_tokens(static_cast<glp_ctx*>(user), ids, lengths, n_seq, max_len, out_dim, out, nullptr);
}

// util.rs:6-29: the first `dim` values divided by their L2 norm (f32, summed in order); a zero
// norm leaves them unchanged
void truncate_mrl(const float* v, int dim, float* out) {
  float ss = 0.f;
  for (int i = 0; i < dim; ++i) ss += v[i] * v[i];
  const float norm = std::sqrt(ss);
  for (int i = 0; i < dim; ++i) out[i] = norm == 0.f ? v[i] : v[i] / norm;
}

}  // namespace

struct glp_engine {
  glp_batch_fn fn = nullptr;
  void* user = nullptr;
  bool model_executor = false;  // fn is glp_embed_tokens: its failures carry glp_last_error()
  int dim = 0;
  int max_batch = 1;
  size_t capacity = 1;
  std::mutex mu;
  std::condition_variable cv_work;   // the worker: a request arrived, or stop
  std::condition_variable cv_space;  // clients: queue space
  std::condition_variable cv_done;   // clients: a batch finished; destroy: last client left
  std::deque<Request*> queue;
  bool stopping = false;
  int active = 0;  // client threads inside glp_engine_embed
  std::thread worker;
  int64_t n_requests = 0, n_batches = 0;
  int largest_batch = 0;

  void run() {
    std::vector<Request*> batch;
    std::vector<int32_t> ids, lengths;
    std::vector<float> rows;
    std::unique_lock<std::mutex> lk(mu);
    while (true) {
      cv_work.wait(lk, [&] { return stopping || !queue.empty(); });
      if (queue.empty()) break;  // stopping and drained
      batch.clear();
      auto drain = [&] {
        while (!queue.empty() && static_cast<int>(batch.size()) < max_batch) {
          batch.push_back(queue.front());
          queue.pop_front();
        }
      };
      drain();
      if (static_cast<int>(batch.size()) < max_batch) {  // coalesce concurrently arriving requests
        lk.unlock();
        std::this_thread::yield();
        lk.lock();
        drain();
      }
      cv_space.notify_all();
      lk.unlock();

      // right-padded batch (pad id 0, never read past each length), one executor call
      const int n = static_cast<int>(batch.size());
      int max_len = 0;
      for (Request* r : batch) max_len = std::max(max_len, r->len);
      ids.assign(static_cast<size_t>(n) * std::max(max_len, 1), 0);
      lengths.resize(n);
      for (int i = 0; i < n; ++i) {
        lengths[i] = batch[i]->len;
        if (batch[i]->len > 0)
          std::memcpy(&ids[static_cast<size_t>(i) * max_len], batch[i]->ids, sizeof(int32_t) * batch[i]->len);
      }
      rows.assign(static_cast<size_t>(n) * dim, 0.f);
      const int rc = fn(user, ids.data(), lengths.data(), n, max_len, dim, rows.data());
      std::string err;
      if (rc != GLP_OK) {
        err = "Batch inference error: " +
              (model_executor ? std::string(glp_last_error()) : "executor returned " + std::to_string(rc));
      }
      for (int i = 0; i < n; ++i) {
        Request* r = batch[i];
        r->rc = rc;
        if (rc != GLP_OK) {
          r->err = err;
          continue;
        }
        const float* row = &rows[static_cast<size_t>(i) * dim];
        if (r->truncate_dim > 0 && r->truncate_dim < dim)
          truncate_mrl(row, r->truncate_dim, r->out);
        else
          std::memcpy(r->out, row, sizeof(float) * dim);
      }

      lk.lock();
      for (Request* r : batch) r->done = true;
      n_requests += n;
      n_batches += 1;
      largest_batch = std::max(largest_batch, n);
      cv_done.notify_all();
    }
  }
};

namespace {

int engine_create(glp_batch_fn fn, void* user, bool model, int dim, int max_batch, int queue_capacity,
                  glp_engine** out) {
  if (!out) {
    glp::set_last_error("out is NULL");
    return GLP_ERR_INVALID_ARG;
  }
  *out = nullptr;
  if (!fn || dim <= 0 || max_batch <= 0 || queue_capacity < 0) {
    glp::set_last_error("engine needs an executor, a positive width and max_batch, queue_capacity >= 0");
    return GLP_ERR_INVALID_ARG;
  }
  auto* e = new glp_engine();
  e->fn = fn;
  e->user = user;
  e->model_executor = model;
  e->dim = dim;
  e->max_batch = max_batch;
  e->capacity = queue_capacity > 0 ? static_cast<size_t>(queue_capacity) : 1024;
  try {
    e->worker = std::thread([e] { e->run(); });
  } catch (const std::exception&) {
    delete e;
    glp::set_last_error("cannot start the engine's worker thread");
    return GLP_ERR_OOM;
  }
  *out = e;
  return GLP_OK;
}

}  // namespace

extern "C" {

int glp_engine_create(glp_ctx* ctx, int max_batch, int queue_capacity, glp_engine** out) {
  if (!ctx) {
    glp::set_last_error("ctx is NULL");
    return GLP_ERR_INVALID_ARG;
  }
  glp_model_info_t info{};
  const int rc = glp_model_info(ctx, &info);
  if (rc != GLP_OK) return rc;
  return engine_create(model_batch, ctx, true, info.embedding_dim, max_batch, queue_capacity, out);
}

int glp_engine_create_with_executor(glp_batch_fn fn, void* user, int embedding_dim, int max_batch,
                                    int queue_capacity, glp_engine** out) {
  return engine_create(fn, user, false, embedding_dim, max_batch, queue_capacity, out);
}

int glp_engine_embed(glp_engine* e, const int32_t* ids, int len, int truncate_dim, float* out) {
  if (!e || (len > 0 && !ids) || !out || len < 0 || truncate_dim < 0) {
    glp::set_last_error("bad engine request (NULL engine or buffer, negative length or dimension)");
    return GLP_ERR_INVALID_ARG;
  }
  Request r;
  r.ids = ids;
  r.len = len;
  r.truncate_dim = truncate_dim;
  r.out = out;
  std::unique_lock<std::mutex> lk(e->mu);
  ++e->active;
  e->cv_space.wait(lk, [&] { return e->stopping || e->queue.size() < e->capacity; });
  if (e->stopping) {
    if (--e->active == 0) e->cv_done.notify_all();
    lk.unlock();
    glp::set_last_error("Inference worker is not running");
    return GLP_ERR_INVALID_ARG;
  }
  e->queue.push_back(&r);
  e->cv_work.notify_one();
  e->cv_done.wait(lk, [&] { return r.done; });
  if (--e->active == 0) e->cv_done.notify_all();
  lk.unlock();
  if (r.rc != GLP_OK) glp::set_last_error(r.err);
  return r.rc;
}

int glp_engine_embed_text(glp_engine* e, const glp_tokenizer* tok, const char* text, size_t text_len, const char* task,
                          const char* title, int truncate_dim, float* out) {
  if (!e || !tok || (text_len && !text) || !out) {
    glp::set_last_error("bad engine text request (NULL engine, tokenizer or buffer)");
    return GLP_ERR_INVALID_ARG;
  }
  if (!glp::valid_utf8(text, text_len) || (task && !glp::valid_utf8(task, std::strlen(task))) ||
      (title && !glp::valid_utf8(title, std::strlen(title)))) {
    glp::set_last_error("not valid UTF-8");
    return GLP_ERR_INVALID_ARG;
  }
  // handlers.rs:88-92 -> MultimodalInput::text -> encode_modality_sequence (tokenizer.rs:454-566)
  std::vector<int32_t> ids;
  const std::string formatted = glp::format_task(task, title, std::string_view(text, text_len));
  const std::string err = glp::tokenize_text(tok, formatted, GLP_TOKENS_SEQUENCE, &ids);
  if (!err.empty()) {
    glp::set_last_error(err);
    return GLP_ERR_INVALID_ARG;
  }
  if (ids.size() > static_cast<size_t>(GLP_DEFAULT_MAX_SEQ_LEN)) {
    glp::set_last_error("Text sequence length (" + std::to_string(ids.size()) +
                        " tokens) exceeds maximum context limit (" + std::to_string(GLP_DEFAULT_MAX_SEQ_LEN) +
                        " tokens)");
    return GLP_ERR_CONTEXT_LIMIT;
  }
  return glp_engine_embed(e, ids.data(), static_cast<int>(ids.size()), truncate_dim, out);
}

int glp_engine_stats(glp_engine* e, int64_t* requests, int64_t* batches, int* largest_batch) {
  if (!e) {
    glp::set_last_error("engine is NULL");
    return GLP_ERR_INVALID_ARG;
  }
  std::lock_guard<std::mutex> lk(e->mu);
  if (requests) *requests = e->n_requests;
  if (batches) *batches = e->n_batches;
  if (largest_batch) *largest_batch = e->largest_batch;
  return GLP_OK;
}

void glp_engine_destroy(glp_engine* e) {
  if (!e) return;
  {
    std::lock_guard<std::mutex> lk(e->mu);
    e->stopping = true;
  }
  e->cv_work.notify_all();
  e->cv_space.notify_all();
  if (e->worker.joinable()) e->worker.join();  // every queued request has been answered
  {
    std::unique_lock<std::mutex> lk(e->mu);  // and every client has left the engine
    e->cv_done.wait(lk, [&] { return e->active == 0; });
  }
  delete e;
}

}  // extern "C"
