// instantiation of the device engine for OrAnd (Int32)
#include "engine_host.cuh"
namespace pp {
extern const Ops ops_orand_i32 = Engine<ORAND, int32_t>::make(ORAND, 2);
}  // namespace pp
