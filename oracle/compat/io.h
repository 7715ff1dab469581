/* Linux stand-in for the MSVC <io.h> calls used by the reference's
   tokenizer persistence (test infrastructure for the oracle build only). */
#ifndef MINIMA_ORACLE_COMPAT_IO_H
#define MINIMA_ORACLE_COMPAT_IO_H
#include <stdio.h>
#include <unistd.h>
static inline int _fileno(FILE* f) { return fileno(f); }
static inline int _commit(int fd) { return fsync(fd); }
#endif
