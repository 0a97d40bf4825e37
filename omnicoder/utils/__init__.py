"""Runtime utilities: logging, performance counters and tracing, environment registry."""
