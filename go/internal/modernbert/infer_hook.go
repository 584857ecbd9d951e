// The lines the device path needs inside the reference's own functions of
// internal/modernbert (infer.go), shown as the small functions they call.
// gpuEnabled is a constant, so without the indecisgpu tag every branch below
// compiles away and the package behaves exactly as before.
//
//	func (m *Model) run(seqs [][]int32, done func(xn []float32, offs []int)) error {   // infer.go:304
//		if gpuEnabled && m.int8 {
//			return m.runGPU(seqs, done)
//		}
//		...
//
//	func (m *Model) EncodeSeqs(seqs [][]int32) ([]float32, error) {                    // infer.go:261
//		if gpuEnabled && m.int8 {
//			return m.encodeSeqsGPU(seqs)
//		}
//		...
//
//	func (m *Model) Invalidate() { ...; m.invalidateGPU() }                             // infer.go:95
//	func (m *Model) SetInt8(on bool) { ...; m.setInt8GPU(on) }                          // infer.go:119
package modernbert

// useGPU reports whether run and EncodeSeqs go to the device for m.
func (m *Model) useGPU() bool { return gpuEnabled && m.int8 }
