// instantiation of the device engine for MaxPlus (Float32, Float64)
#include "engine_host.cuh"
namespace pp {
extern const Ops ops_maxplus_f32 = Engine<MAXPLUS, float>::make(MAXPLUS, 0);
extern const Ops ops_maxplus_f64 = Engine<MAXPLUS, double>::make(MAXPLUS, 1);
}  // namespace pp
