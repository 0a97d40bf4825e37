"""Export / compatibility: GGUF files, ONNX decode-step graphs, mobile packages
(off the benchmarked path)."""
