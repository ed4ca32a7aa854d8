// seeded.cpp -- TEST INFRASTRUCTURE ONLY.
//
// The reference's tests draw their inputs from std::mt19937 through
// std::normal_distribution<float> (src/appnnc/tests.cpp:2452-2453). The
// seeded synthetic configurations use the same generator, so the checker can
// reproduce a configuration from its seed alone. One handle is one stream:
// drawing q, then k, then v, then gamma from it fixes the order.
#include "oracle.h"

#include <random>

namespace
{
	// The normal distribution is kept with the engine: it draws values in
	// pairs and hands out the second on the next call, so a fresh one per
	// call would give a different stream from the reference's single `nd`.
	struct rng_state
	{
		std::mt19937 gen;
		std::normal_distribution<float> nd{0.0f, 1.0f};
		explicit rng_state(uint32_t seed) : gen(seed) {}
	};
}

extern "C" void* orc_rng_new(uint32_t seed) { return new rng_state(seed); }

extern "C" void orc_rng_normal(void* rng, float* out, size_t n, float mean, float stddev)
{
	auto* r = static_cast<rng_state*>(rng);
	for (size_t i = 0; i < n; ++i) out[i] = r->nd(r->gen) * stddev + mean;
}

extern "C" void orc_rng_uniform(void* rng, float* out, size_t n, float lo, float hi)
{
	auto* r = static_cast<rng_state*>(rng);
	std::uniform_real_distribution<float> ud(lo, hi);
	for (size_t i = 0; i < n; ++i) out[i] = ud(r->gen);
}

extern "C" void orc_rng_free(void* rng) { delete static_cast<rng_state*>(rng); }
