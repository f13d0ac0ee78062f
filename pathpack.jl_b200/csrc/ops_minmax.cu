// instantiation of the device engine for MinMax (Float32, Float64)
#include "engine_host.cuh"
namespace pp {
extern const Ops ops_minmax_f32 = Engine<MINMAX, float>::make(MINMAX, 0);
extern const Ops ops_minmax_f64 = Engine<MINMAX, double>::make(MINMAX, 1);
}  // namespace pp
