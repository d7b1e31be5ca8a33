/* Forced include for compiling the reference's CPU sources with g++ on Linux
 * (oracle/Makefile). The reference targets MSVC; these standard headers are
 * the only ones its tensor sources rely on transitively there. */
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <limits>
