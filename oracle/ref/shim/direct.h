/* Build shim for compiling the reference's Stage 2e sources on Linux: the
 * reference calls the Windows-only _mkdir from <direct.h> when it writes a
 * checkpoint directory.  Semantics unchanged (mkdir with mode 0755). */
#pragma once
#include <sys/stat.h>
#define _mkdir(d) mkdir((d), 0755)
