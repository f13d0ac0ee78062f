// instantiation of the device engine for PlusProd (Float32, Float64)
#include "engine_host.cuh"
namespace pp {
extern const Ops ops_plusprod_f32 = Engine<PLUSPROD, float>::make(PLUSPROD, 0);
extern const Ops ops_plusprod_f64 = Engine<PLUSPROD, double>::make(PLUSPROD, 1);
}  // namespace pp
