"""CPU oracle of the sampling path (test infrastructure only; see sampling_ref.h)."""
