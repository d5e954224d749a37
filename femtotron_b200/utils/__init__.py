"""Runtime utilities: distributed init, device timing, clock sampling, metrics."""
