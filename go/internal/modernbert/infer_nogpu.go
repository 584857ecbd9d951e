//go:build !indecisgpu

// Without the indecisgpu tag the package keeps its CPU path; these stubs let
// the hooks in infer_hook.go compile away.
package modernbert

const gpuEnabled = false

func (m *Model) runGPU(seqs [][]int32, done func(xn []float32, offs []int)) error {
	panic("modernbert: built without indecisgpu")
}

func (m *Model) encodeSeqsGPU(seqs [][]int32) ([]float32, error) {
	panic("modernbert: built without indecisgpu")
}

func (m *Model) invalidateGPU() {}

func (m *Model) setInt8GPU(on bool) {}
