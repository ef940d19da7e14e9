/* rpg_engine.h -- the engine's public C ABI (ten functions).
 *
 * Drop-in replacement for the reference's include/rpg_engine.h:46-117 and
 * src/rpg_engine.def:11-20: the same ten symbols, argument meanings, ownership
 * and error behaviour, so existing Python ctypes and Unity P/Invoke hosts bind
 * to librpg_engine_b200.so unchanged.
 *
 * Handles: >= 0 valid, < 0 failure (message in rpg_engine_last_error(),
 * thread-local, not to be freed).  Handles are never reused.  Strings returned
 * by the engine are freed with rpg_engine_free.  One generate at a time per
 * session; sessions on different devices may generate concurrently.
 */
#ifndef RPG_ENGINE_H
#define RPG_ENGINE_H

#include <stdint.h>

#if defined(_WIN32)
#if defined(RPG_ENGINE_BUILD)
#define RPG_API __declspec(dllexport)
#else
#define RPG_API
#endif
#elif defined(__GNUC__)
#define RPG_API __attribute__((visibility("default")))
#else
#define RPG_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define RPG_ENGINE_OK 0

/* Engine version string, e.g. "0.1.0" (reference: rpg_engine.h:52). */
RPG_API const char* rpg_engine_version(void);

/* Last error of the calling thread; valid until the next call (rpg_engine.h:55). */
RPG_API const char* rpg_engine_last_error(void);

/* Loads a GGUF model.  config_json (may be NULL): {"context": N, "device": D};
 * "device" is an addition of this engine (default 0).  Returns a model handle
 * or a negative value (rpg_engine.h:62). */
RPG_API int32_t rpg_engine_load_model(const char* model_path, const char* config_json);

/* Unloads a model and every session on it; an invalid handle is a no-op. */
RPG_API void rpg_engine_unload_model(int32_t model);

/* Creates a session (own KV cache).  session_json (may be NULL): {"max_seq",
 * "max_tokens", "temperature", "seed", "stop"} (src/engine.cc:315-391). */
RPG_API int32_t rpg_engine_session_create(int32_t model, const char* session_json);

/* Destroys a session and frees its KV cache; an invalid handle is a no-op. */
RPG_API void rpg_engine_session_destroy(int32_t session);

/* Clears the KV cache and cached prompt, keeps the configuration; 0 = OK. */
RPG_API int32_t rpg_engine_session_reset(int32_t session);

/* Runs one generation.  Request JSON: {"messages": [...], "tools": [...],
 * "max_tokens", "temperature", "top_p", "stop", "seed", "enable_thinking"};
 * response JSON: {"text", "tool_calls", "finish_reason", "usage"}
 * (rpg_engine.h:83-107, src/engine.cc:429-615).  Returns a new string to be
 * released with rpg_engine_free, or NULL on failure. */
RPG_API char* rpg_engine_generate(int32_t session, const char* request_json);

/* Frees a string returned by the engine. */
RPG_API void rpg_engine_free(char* buf);

/* Model metadata JSON (src/engine.cc:619-665); free with rpg_engine_free. */
RPG_API char* rpg_engine_model_info(int32_t model);

#ifdef __cplusplus
}
#endif

#endif /* RPG_ENGINE_H */
