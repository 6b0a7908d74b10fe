// Tensor-core screen for top-1 (tcgen05). Placeholder until the screen lands:
// every call takes the exact SIMT path.
#include "engine.h"

namespace eb {

struct Fp16Copy {};

bool top1_screen_supported(eb_engine*, const Top1Args&) { return false; }
void top1_screen(eb_engine* e, const Top1Args& a, eb_buf*) { top1_exact(e, a); }
void drop_f16(eb_buf* b) {
  if (b && b->f16) {
    delete b->f16;
    b->f16 = nullptr;
  }
}

}  // namespace eb
