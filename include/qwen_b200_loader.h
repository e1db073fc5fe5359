/* Native safetensors checkpoint reader for the Qwen3-0.6B weights.
 *
 * Replaces the Hugging Face model instantiation inside upstream
 * load_weights (Model/Qwen06B_architecture.py:97-174: AutoModelForCausalLM
 * .from_pretrained(model_name, torch_dtype=torch.float16) followed by
 * model.state_dict()).  Upstream reads the checkpoint through transformers and
 * casts every tensor to fp16 on the way; this reader parses the safetensors
 * header itself, streams the tensor bytes from the file through pinned host
 * buffers into device memory and casts BF16 / F32 to F16 on the device with
 * round-to-nearest-even (bit-identical to torch's .to(torch.float16)).
 *
 * File format (safetensors): 8-byte little-endian header length N, N bytes of
 * JSON {name: {"dtype", "shape", "data_offsets": [begin, end]}, ...,
 * "__metadata__": {...}}, then the data; offsets count from the end of the
 * header.  Tensors are row-major and tightly packed.
 *
 * Every function returns 0 on success or an error code; the message is
 * available through qwen_b200_last_error (include/qwen_b200.h).  Handles are
 * not thread-safe; one handle may be used from one thread at a time.
 */
#ifndef QWEN_B200_LOADER_H
#define QWEN_B200_LOADER_H

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element types of a safetensors file that the reader understands. */
enum {
  QWEN_ST_F16 = 0,
  QWEN_ST_BF16 = 1,
  QWEN_ST_F32 = 2,
  QWEN_ST_OTHER = 3 /* listed by qwen_b200_st_info, rejected by the loads */
};

typedef struct QwenStFile QwenStFile;

/* Opens `path` and parses and validates its header (every tensor lies inside
 * the file and its byte size equals numel x element size).  No CUDA call. */
int qwen_b200_st_open(const char *path, QwenStFile **out);
void qwen_b200_st_close(QwenStFile *f);

int qwen_b200_st_num_tensors(const QwenStFile *f);
/* Index of the tensor called `name`, or -1. */
int qwen_b200_st_find(const QwenStFile *f, const char *name);
/* Tensor i: its name (valid until close), element type, rank (<= 8), shape and
 * byte size. */
int qwen_b200_st_info(const QwenStFile *f, int i, const char **name, int *dtype, int *ndim,
                      long long shape[8], long long *nbytes);
/* Value of key `key` in "__metadata__", or NULL. */
const char *qwen_b200_st_metadata(const QwenStFile *f, const char *key);

/* Raw bytes of tensor i into host memory (`cap` bytes available).  No CUDA. */
int qwen_b200_st_read_host(const QwenStFile *f, int i, void *dst, long long cap);

/* Tensor i as fp16 into device memory at `dst` (numel x 2 bytes, 16-byte
 * aligned), enqueued on `stream`; BF16 and F32 are converted on the device.
 * The host side reuses two pinned 16 MiB buffers and one device staging
 * buffer owned by the handle; the call returns once every chunk is enqueued,
 * and the caller synchronises `stream` before reading `dst`.  Closing the
 * handle waits for its copies in flight. */
int qwen_b200_st_load_f16(QwenStFile *f, int i, void *dst, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* QWEN_B200_LOADER_H */
