"""Command-line tools: training orchestration, expert-parallel launcher, HTTP server."""
