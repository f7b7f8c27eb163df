"""CPU oracle of the paged KV store and batch index build (test infrastructure only)."""
