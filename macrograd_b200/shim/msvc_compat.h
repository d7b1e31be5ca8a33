/* Forced include for compiling the reference's sources with g++ on Linux in
 * the drop-in build (Makefile in this directory). The reference targets MSVC;
 * besides standard headers its nn.cpp and model headers use two of MSVC's
 * bounds-checked CRT calls, given here with their documented meaning. */
#pragma once
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <limits>

/* copies src (with its terminator) into dst of `size` bytes; 0 on success */
static inline int strcpy_s(char* dst, size_t size, const char* src)
{
    if (!dst || !src || size == 0) return 22;
    const size_t n = strlen(src);
    if (n >= size) {
        dst[0] = '\0';
        return 34;
    }
    memcpy(dst, src, n + 1);
    return 0;
}

/* opens `path`; *f is NULL on failure; 0 on success */
static inline int fopen_s(FILE** f, const char* path, const char* mode)
{
    if (!f) return 22;
    *f = fopen(path, mode);
    return *f ? 0 : 2;
}
