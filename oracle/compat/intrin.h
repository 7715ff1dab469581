/* Empty stand-in for MSVC <intrin.h>; the reference only uses its
   intrinsics under _MSC_VER, where gcc builtins are used otherwise. */
#ifndef MINIMA_ORACLE_COMPAT_INTRIN_H
#define MINIMA_ORACLE_COMPAT_INTRIN_H
#endif
