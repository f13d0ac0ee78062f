// instantiation of the device engine for MaxMin (Float32, Float64)
#include "engine_host.cuh"
namespace pp {
extern const Ops ops_maxmin_f32 = Engine<MAXMIN, float>::make(MAXMIN, 0);
extern const Ops ops_maxmin_f64 = Engine<MAXMIN, double>::make(MAXMIN, 1);
}  // namespace pp
