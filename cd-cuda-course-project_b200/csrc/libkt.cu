// libkt.cu — the default library: every kernel family with its default
// (tuned) template parameters.
#include "kt_entry.cuh"
