// Internal: the thread-local error slot behind qwen_b200_last_error(), shared
// by every translation unit of libqwen_b200.so (defined in decode.cu).
#pragma once
extern "C" {
void qb200_clear_error(void);
int qb200_set_error(int code, const char *msg);
}
