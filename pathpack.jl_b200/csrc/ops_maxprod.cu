// instantiation of the device engine for MaxProd (Float32, Float64)
#include "engine_host.cuh"
namespace pp {
extern const Ops ops_maxprod_f32 = Engine<MAXPROD, float>::make(MAXPROD, 0);
extern const Ops ops_maxprod_f64 = Engine<MAXPROD, double>::make(MAXPROD, 1);
}  // namespace pp
