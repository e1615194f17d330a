"""CPU oracle of the KV-cached decode path — test infrastructure only (see oracle.h)."""
