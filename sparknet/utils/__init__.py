"""Device timing, clock sampling and environment helpers (shared by bench, probe, tests)."""
