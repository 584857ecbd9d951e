//go:build indecisgpu

// The root package's side of the device path (github.com/bornholm/indecis):
// the memory-mapped embedding table hands its stored arrays to the device
// (modernbert.StoredTable), and Load gives the encoder the model file's raw
// layer tensors (modernbert.SetStoredSource), so neither the 393 MB float32
// table nor float32 layer matrices are built on the host.
package indecis

import (
	"github.com/bornholm/indecis/internal/modernbert"
	"github.com/bornholm/indecis/safetensors"
)

// Stored implements modernbert.StoredTable (embeddings.go:9-68): the int8
// rows and scales, or the bf16 rows with the exact float32 rows by rank.
func (e *mappedEmbeddings) Stored() (bf16 []byte, exactIDs []int32, exactRows []byte, i8 []byte, scale []float32) {
	if e.i8 != nil {
		return nil, nil, nil, e.i8, e.scale
	}
	ids := make([]int32, len(e.exact))
	for id, rank := range e.exact {
		ids[rank] = id
	}
	return e.bf16, ids, e.f32, nil, nil
}

var _ modernbert.StoredTable = (*mappedEmbeddings)(nil)

// gpuStoredSource is called by Load (model.go:719, beside SetCompact) with
// the opened model file.
func gpuStoredSource(enc *modernbert.Model, f *safetensors.File) {
	enc.SetStoredSource(func(name string) (modernbert.RawTensor, bool) {
		dtype, _, raw, ok := f.Raw(name)
		if !ok || len(raw) == 0 {
			return modernbert.RawTensor{}, false
		}
		return modernbert.RawTensor{DType: dtype, Data: raw}, true
	})
}
