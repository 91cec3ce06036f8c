package main

import "math/rand"

// Accelerator hook for the examples' sample step, consulted first by sample
// (sample_hook.diff: _example/gpt2/main.go:69, _example/qwen/main.go:115).
// Nil in a plain build, so the Go body runs unchanged; example_sample_cuda.go
// sets it in `-tags cuda` builds. It returns done = true with the token.
var sampleHook func(logits []float32, temp float64, rng *rand.Rand) (id int, done bool)
