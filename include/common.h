/*
 * common.h -- shared scalar types and compile-time limits of the llamini C API.
 *
 * Drop-in counterpart of llamini.cpp common.h:1-33. The typedef names, their
 * widths and the macro values are part of the caller-visible ABI (every struct
 * in gguf.h/model.h/kv_cache.h/tensor.h/gpt2.h is laid out with them), so they
 * are kept identical. The system headers are included here too because callers
 * of the reference API (its main.c) rely on them arriving through this header.
 */
#ifndef COMMON_H
#define COMMON_H

#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>
#include <unistd.h>
#include <sys/types.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <fcntl.h>
#include <time.h>
#include <ctype.h>
#include <assert.h>

/* Limits (common.h:17-21). MAX_SEQ_LEN caps every model's context length. */
#define MAX_DIM        4096
#define MAX_SEQ_LEN    2048
#define MAX_TOKEN_LEN  256
#define MAX_PROMPT_LEN 1024
#define EPS            1e-8f

/* Fixed-width aliases (common.h:23-29). */
typedef float              f32;
typedef unsigned char      u8;
typedef signed char        i8;
typedef unsigned short     u16;
typedef unsigned int       u32;
typedef int                i32;
typedef unsigned long long u64;

/* Default special token ids (common.h:31-32). */
#define TOKEN_BOS  1
#define TOKEN_EOS  2

#endif
