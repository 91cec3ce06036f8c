package tensai

// Accelerator hooks for the quantized MatVec, consulted by QMatrix.MatVec and
// Q4Matrix.MatVec after their shape checks (matvec_hook.diff). Nil in a
// plain build, so the CPU bodies run unchanged; quant_cuda.go sets them in
// `-tags cuda` builds. A hook returns done = true when it produced out (or
// the error to report).
var (
	q8MatVecHook func(q *QMatrix, x, out []Float) (done bool, err error)
	q4MatVecHook func(q *Q4Matrix, x, out []Float) (done bool, err error)
)
