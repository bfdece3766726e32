// Ring attention over NCCL (attnax/kernels/attention.py:540-691).
//
// The reference rotates K/V with two lax.ppermute calls per step
// (:673-674) and carries (m, l, o) through a lax.scan (:678-682).  Here one
// process drives one GPU; this file owns the NCCL communicator that plays
// the role of the bound device axis (axis_size / axis_index, :604-617).
#include <nccl.h>

#include "attn_common.cuh"

namespace attnb200 {
namespace ring {

struct Comm {
  ncclComm_t comm = nullptr;
  int nranks = 0, rank = 0;
};

}  // namespace ring
}  // namespace attnb200
