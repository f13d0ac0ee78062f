// instantiation of the device engine for MinPlus (Float32, Float64, Int32)
#include "engine_host.cuh"
namespace pp {
extern const Ops ops_minplus_f32 = Engine<MINPLUS, float>::make(MINPLUS, 0);
extern const Ops ops_minplus_f64 = Engine<MINPLUS, double>::make(MINPLUS, 1);
extern const Ops ops_minplus_i32 = Engine<MINPLUS, int32_t>::make(MINPLUS, 2);
}  // namespace pp
