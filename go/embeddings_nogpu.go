//go:build !indecisgpu

package indecis

import (
	"github.com/bornholm/indecis/internal/modernbert"
	"github.com/bornholm/indecis/safetensors"
)

func gpuStoredSource(enc *modernbert.Model, f *safetensors.File) {}
