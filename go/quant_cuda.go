//go:build cuda && linux

// Package tensai, CUDA build: QMatrix.MatVec and Q4Matrix.MatVec run on a
// B200 through libtensai_cuda.so (include/tensai_cuda.h), bound with purego
// the way wgpu.go binds wgpu-native, so no cgo is needed. Copy this file and
// quant_hooks.go into the tensai package and apply matvec_hook.diff
// (quant.go:77-81, quant4.go:93-97); build with `go build -tags cuda`.
//
// Weights are uploaded once per matrix (tq_q8_upload / tq_q4_upload take the
// exported Q and Scale slices as they are) and stay resident in HBM until
// FreeCUDA. A cuda build whose library cannot be loaded fails every MatVec
// with that error: there is no silent CPU fallback.
package tensai

import (
	"fmt"
	"os"
	"runtime"
	"sync"
	"unsafe"

	"github.com/ebitengine/purego"
)

// tqABIVersion is TQ_ABI_VERSION of include/tensai_cuda.h.
const tqABIVersion = 1

var (
	cudaOnce sync.Once
	cudaErr  error

	tqVersion   func() int32
	tqLastError func() uintptr
	tqQ8Upload  func(q, scale unsafe.Pointer, rows, cols int32, h *uint64) int32
	tqQ4Upload  func(q, scale unsafe.Pointer, rows, cols int32, h *uint64) int32
	tqMatVec    func(h uint64, x unsafe.Pointer, xLen uintptr, out unsafe.Pointer, outLen uintptr) int32
	tqFree      func(h uint64) int32

	// Device handles of uploaded matrices, keyed by the Go matrix, so the
	// exported QMatrix / Q4Matrix fields stay as they are.
	cudaMu      sync.Mutex
	cudaHandles = map[unsafe.Pointer]uint64{}
)

func loadCUDA() error {
	cudaOnce.Do(func() {
		name := os.Getenv("TENSAI_CUDA_LIB")
		if name == "" {
			name = "libtensai_cuda.so"
		}
		lib, err := purego.Dlopen(name, purego.RTLD_NOW|purego.RTLD_GLOBAL)
		if err != nil {
			cudaErr = fmt.Errorf("tensai: cannot load %s (set TENSAI_CUDA_LIB): %w", name, err)
			return
		}
		purego.RegisterLibFunc(&tqVersion, lib, "tq_version")
		if v := tqVersion(); v != tqABIVersion {
			cudaErr = fmt.Errorf("tensai: %s has ABI %d, want %d", name, v, tqABIVersion)
			return
		}
		purego.RegisterLibFunc(&tqLastError, lib, "tq_last_error")
		purego.RegisterLibFunc(&tqQ8Upload, lib, "tq_q8_upload")
		purego.RegisterLibFunc(&tqQ4Upload, lib, "tq_q4_upload")
		purego.RegisterLibFunc(&tqMatVec, lib, "tq_matvec")
		purego.RegisterLibFunc(&tqFree, lib, "tq_free")
	})
	return cudaErr
}

// cudaCString copies the library's NUL-terminated message into a Go string.
func cudaCString(p uintptr) string {
	if p == 0 {
		return ""
	}
	ptr := *(*unsafe.Pointer)(unsafe.Pointer(&p)) // a C pointer, not a Go object
	var out []byte
	for i := 0; ; i++ {
		c := *(*byte)(unsafe.Add(ptr, i))
		if c == 0 {
			return string(out)
		}
		out = append(out, c)
	}
}

func cudaError() error { return fmt.Errorf("%s", cudaCString(tqLastError())) }

// handleFor uploads a matrix's codes and scales on its first MatVec and
// returns the device handle of later calls.
func handleFor(key unsafe.Pointer, bits int, q, scale unsafe.Pointer, rows, cols int) (uint64, error) {
	cudaMu.Lock()
	defer cudaMu.Unlock()
	if h, ok := cudaHandles[key]; ok {
		return h, nil
	}
	up := tqQ8Upload
	if bits == 4 {
		up = tqQ4Upload
	}
	var h uint64
	if up(q, scale, int32(rows), int32(cols), &h) != 0 {
		return 0, cudaError()
	}
	cudaHandles[key] = h
	return h, nil
}

// cudaMatVec is the body of both hooks: the shape was checked by MatVec.
func cudaMatVec(key unsafe.Pointer, bits int, q, scale unsafe.Pointer, rows, cols int, x, out []Float) error {
	if err := loadCUDA(); err != nil {
		return err
	}
	if rows == 0 || cols == 0 {
		for i := range out {
			out[i] = 0
		}
		return nil
	}
	h, err := handleFor(key, bits, q, scale, rows, cols)
	if err != nil {
		return err
	}
	rc := tqMatVec(h, unsafe.Pointer(&x[0]), uintptr(len(x)), unsafe.Pointer(&out[0]), uintptr(len(out)))
	runtime.KeepAlive(x)
	runtime.KeepAlive(out)
	if rc != 0 {
		return cudaError()
	}
	return nil
}

func init() {
	q8MatVecHook = func(m *QMatrix, x, out []Float) (bool, error) {
		var q, s unsafe.Pointer
		if len(m.Q) > 0 {
			q, s = unsafe.Pointer(&m.Q[0]), unsafe.Pointer(&m.Scale[0])
		}
		err := cudaMatVec(unsafe.Pointer(m), 8, q, s, m.Rows, m.Cols, x, out)
		runtime.KeepAlive(m)
		return true, err
	}
	q4MatVecHook = func(m *Q4Matrix, x, out []Float) (bool, error) {
		var q, s unsafe.Pointer
		if len(m.Q) > 0 {
			q, s = unsafe.Pointer(&m.Q[0]), unsafe.Pointer(&m.Scale[0])
		}
		err := cudaMatVec(unsafe.Pointer(m), 4, q, s, m.Rows, m.Cols, x, out)
		runtime.KeepAlive(m)
		return true, err
	}
}

// FreeCUDA releases the device copy of a *QMatrix or *Q4Matrix (explicit,
// like GPUTensor.Free, wgputensor.go:676-686; a second call is a no-op).
// A matrix whose Q or Scale is changed after its first MatVec must be freed
// first: the device copy is made once.
func FreeCUDA(m any) {
	var key unsafe.Pointer
	switch v := m.(type) {
	case *QMatrix:
		key = unsafe.Pointer(v)
	case *Q4Matrix:
		key = unsafe.Pointer(v)
	default:
		return
	}
	cudaMu.Lock()
	defer cudaMu.Unlock()
	if h, ok := cudaHandles[key]; ok {
		tqFree(h)
		delete(cudaHandles, key)
	}
}
