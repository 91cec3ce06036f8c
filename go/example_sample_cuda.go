//go:build cuda && linux

// Package main, CUDA build of an example: sample (main.go:69-105 of
// _example/gpt2, main.go:115-150 of _example/qwen) runs on a B200 through
// tq_sample in libtensai_cuda.so (include/tensai_cuda.h), bound with purego.
// Copy this file and example_sample_hooks.go into the example's directory and
// apply sample_hook.diff; build with `go build -tags cuda`. The draw is the
// example's own rng.Float64(), taken only when temp > 0 as the Go body takes
// it, so a seeded run draws the same stream. A library that cannot be loaded
// panics with its error: there is no silent fallback to the Go body.
package main

import (
	"fmt"
	"math/rand"
	"os"
	"runtime"
	"sync"
	"unsafe"

	"github.com/ebitengine/purego"
)

var (
	sampleOnce   sync.Once
	sampleErr    error
	tqSample     func(logits unsafe.Pointer, n int32, temp float64, u float64, token *int32) int32
	tqLastErrorS func() uintptr
)

func loadSample() error {
	sampleOnce.Do(func() {
		name := os.Getenv("TENSAI_CUDA_LIB")
		if name == "" {
			name = "libtensai_cuda.so"
		}
		lib, err := purego.Dlopen(name, purego.RTLD_NOW|purego.RTLD_GLOBAL)
		if err != nil {
			sampleErr = fmt.Errorf("tensai: cannot load %s (set TENSAI_CUDA_LIB): %w", name, err)
			return
		}
		purego.RegisterLibFunc(&tqSample, lib, "tq_sample")
		purego.RegisterLibFunc(&tqLastErrorS, lib, "tq_last_error")
	})
	return sampleErr
}

// lastError copies the library's NUL-terminated message.
func lastError() string {
	p := tqLastErrorS()
	if p == 0 {
		return ""
	}
	ptr := *(*unsafe.Pointer)(unsafe.Pointer(&p)) // a C pointer, not a Go object
	var b []byte
	for i := 0; ; i++ {
		c := *(*byte)(unsafe.Add(ptr, i))
		if c == 0 {
			return string(b)
		}
		b = append(b, c)
	}
}

func init() {
	sampleHook = func(logits []float32, temp float64, rng *rand.Rand) (int, bool) {
		if err := loadSample(); err != nil {
			panic(err)
		}
		u := 0.0
		if temp > 0 {
			u = rng.Float64()
		}
		var tok int32
		rc := tqSample(unsafe.Pointer(&logits[0]), int32(len(logits)), temp, u, &tok)
		runtime.KeepAlive(logits)
		if rc != 0 {
			panic(fmt.Errorf("%s", lastError()))
		}
		return int(tok), true
	}
}
