//go:build indecisgpu

// The int8 inference path of package modernbert on NVIDIA B200 GPUs, through
// the C ABI of libindecis_b200 (include/indecis_b200.h).
//
// This file belongs in github.com/bornholm/indecis/internal/modernbert. With
// the build tag indecisgpu, run (infer.go:304) sends int8 inference to the
// device (see the hook in infer_hook.go); without the tag the package is
// unchanged. There is no CPU fallback in a GPU build: a missing device is an
// error at first use.
//
// Devices: every sm_100 GPU the process sees, or the ordinals listed in
// INDECIS_GPUS ("0,1,2,3"). With several, each call's sequences are split
// into contiguous cost-balanced ranges, one per GPU (ig_model_create_multi),
// and every range lands in its slice of the output.
//
// Weights: when the model file's raw tensors are available
// (SetStoredSource, called by the root package's Load), the layer tensors go
// to the devices in their stored dtype (bf16 checkpoints: half the bytes) and
// the embedding table as stored (bf16 + exact rows, or int8 + scales);
// otherwise the float32 Params are used.
package modernbert

/*
#cgo CFLAGS: -I${SRCDIR}/../../third_party/indecis_b200/include
#cgo LDFLAGS: -L${SRCDIR}/../../third_party/indecis_b200 -lindecis_b200 -Wl,-rpath,${SRCDIR}/../../third_party/indecis_b200
#include <stdlib.h>
#include "indecis_b200.h"
*/
import "C"

import (
	"errors"
	"fmt"
	"os"
	"runtime"
	"strconv"
	"strings"
	"sync"
	"unsafe"
)

const gpuEnabled = true

// RawTensor is a tensor as the model file stores it: DType "F32", "BF16",
// "F16" or "I8" (safetensors.File.Raw) and its little-endian bytes.
type RawTensor struct {
	DType string
	Data  []byte
}

// StoredSource returns a tensor of the model file by name, undecoded.
type StoredSource func(name string) (RawTensor, bool)

// StoredTable is an embedding table that can hand its stored arrays to the
// device (the root package's mappedEmbeddings implements it): bf16 rows as
// little-endian bytes plus float32 exact rows for the listed ids, or int8
// rows and a scale per row.
type StoredTable interface {
	Stored() (bf16 []byte, exactIDs []int32, exactRows []byte, i8 []byte, scale []float32)
}

type gpuState struct {
	mu     sync.Mutex
	h      *C.ig_model
	err    error
	stored StoredSource
}

var gpuStates sync.Map // *Model -> *gpuState

func (m *Model) gpuState() *gpuState {
	v, _ := gpuStates.LoadOrStore(m, &gpuState{})
	return v.(*gpuState)
}

// SetStoredSource gives the device path the model file's raw tensors, so
// that the weights are uploaded as stored rather than decoded to float32.
func (m *Model) SetStoredSource(src StoredSource) {
	g := m.gpuState()
	g.mu.Lock()
	g.stored = src
	g.mu.Unlock()
}

func gpuDevices() ([]C.int32_t, error) {
	if s := strings.TrimSpace(os.Getenv("INDECIS_GPUS")); s != "" {
		var ds []C.int32_t
		for _, f := range strings.Split(s, ",") {
			d, err := strconv.Atoi(strings.TrimSpace(f))
			if err != nil {
				return nil, fmt.Errorf("modernbert: gpu: INDECIS_GPUS: %v", err)
			}
			ds = append(ds, C.int32_t(d))
		}
		return ds, nil
	}
	var n C.int32_t
	C.ig_device_count(&n)
	if n == 0 {
		return nil, errors.New("modernbert: gpu: no sm_100 device")
	}
	ds := make([]C.int32_t, n)
	for i := range ds {
		ds[i] = C.int32_t(i)
	}
	return ds, nil
}

func lastError() error { return errors.New(C.GoString(C.ig_last_error())) }

// gpu returns the device model, created on first use (and again after
// Invalidate).
func (m *Model) gpu() (*C.ig_model, error) {
	g := m.gpuState()
	g.mu.Lock()
	defer g.mu.Unlock()
	if g.h == nil && g.err == nil {
		g.h, g.err = m.createGPU(g.stored)
	}
	return g.h, g.err
}

// invalidateGPU drops the device copy: Invalidate (infer.go:95) calls it
// when the weights change.
func (m *Model) invalidateGPU() {
	g := m.gpuState()
	g.mu.Lock()
	defer g.mu.Unlock()
	if g.h != nil {
		C.ig_model_destroy(g.h)
	}
	g.h, g.err = nil, nil
}

// cArray is a C array of n elements of T (cgo: pointers to Go memory may
// not be stored in Go memory that is passed to C).
func cArray[T any](n int) []T {
	var t T
	p := C.calloc(C.size_t(n), C.size_t(unsafe.Sizeof(t)))
	return unsafe.Slice((*T)(p), n)
}

func cFree[T any](s []T) { C.free(unsafe.Pointer(unsafe.SliceData(s))) }

func (m *Model) config() C.ig_config {
	c := C.ig_config{
		vocab: C.int32_t(m.Cfg.Vocab), hidden: C.int32_t(m.Cfg.Hidden), layers: C.int32_t(m.Cfg.Layers),
		heads: C.int32_t(m.Cfg.Heads), intermediate: C.int32_t(m.Cfg.Intermediate),
		global_every: C.int32_t(m.Cfg.GlobalEvery), local_attention: C.int32_t(m.Cfg.LocalAttention),
		norm_eps: C.double(m.Cfg.NormEps), global_theta: C.double(m.Cfg.GlobalTheta),
		local_theta: C.double(m.Cfg.LocalTheta), simd_lanes: 8,
	}
	if m.Cfg.CLS() {
		c.pooling = C.IG_POOL_CLS
	}
	return c
}

var dtypes = map[string]C.int32_t{"F32": C.IG_DT_F32, "BF16": C.IG_DT_BF16, "F16": C.IG_DT_F16, "I8": C.IG_DT_I8}

func (m *Model) createGPU(stored StoredSource) (*C.ig_model, error) {
	if err := m.Cfg.validate(); err != nil {
		return nil, err
	}
	devs, err := gpuDevices()
	if err != nil {
		return nil, err
	}
	var pin runtime.Pinner // Go memory handed to C stays pinned for the call only
	defer pin.Unpin()
	f32 := func(s []float32) unsafe.Pointer {
		if len(s) == 0 {
			return nil
		}
		pin.Pin(&s[0])
		return unsafe.Pointer(&s[0])
	}
	cfg := m.config()
	L := len(m.Layers)
	var h *C.ig_model
	if stored != nil {
		// The layer tensors as stored; the norms Load has already decoded.
		views := make([][]C.ig_tensor, 6)
		for i := range views {
			views[i] = cArray[C.ig_tensor](L)
			defer cFree(views[i])
		}
		raw := func(p *Param) (C.ig_tensor, error) {
			t, ok := stored(p.Name)
			if !ok {
				if p.W == nil {
					return C.ig_tensor{}, fmt.Errorf("modernbert: tensor %s missing", p.Name)
				}
				return C.ig_tensor{dtype: C.IG_DT_F32, data: f32(p.W)}, nil
			}
			dt, ok := dtypes[t.DType]
			if !ok {
				return C.ig_tensor{}, fmt.Errorf("modernbert: %s: unsupported dtype %s", p.Name, t.DType)
			}
			pin.Pin(&t.Data[0])
			return C.ig_tensor{dtype: dt, data: unsafe.Pointer(&t.Data[0])}, nil
		}
		for l, Ly := range m.Layers {
			for i, p := range []*Param{Ly.AttnNorm, Ly.Wqkv, Ly.Wo, Ly.MLPNorm, Ly.Wi, Ly.WoMLP} {
				if p == nil { // layer 0 has no attention norm
					continue
				}
				if views[i][l], err = raw(p); err != nil {
					return nil, err
				}
			}
		}
		w := C.ig_stored_weights{
			emb_norm:   C.ig_tensor{dtype: C.IG_DT_F32, data: f32(m.EmbNorm.W)},
			final_norm: C.ig_tensor{dtype: C.IG_DT_F32, data: f32(m.FinalNorm.W)},
			attn_norm:  &views[0][0], wqkv: &views[1][0], wo: &views[2][0],
			mlp_norm: &views[3][0], wi: &views[4][0], wo_mlp: &views[5][0],
		}
		if C.ig_model_create_stored_multi(&cfg, &w, &devs[0], C.int32_t(len(devs)), &h) != C.IG_OK {
			return nil, fmt.Errorf("modernbert: gpu: %v", lastError())
		}
	} else {
		m.restoreWeights() // the float32 layer matrices (SetCompact may have freed them)
		ptrs := make([][]*C.float, 6)
		for i := range ptrs {
			ptrs[i] = cArray[*C.float](L)
			defer cFree(ptrs[i])
		}
		for l, Ly := range m.Layers {
			for i, p := range []*Param{Ly.AttnNorm, Ly.Wqkv, Ly.Wo, Ly.MLPNorm, Ly.Wi, Ly.WoMLP} {
				if p != nil {
					ptrs[i][l] = (*C.float)(f32(p.W))
				}
			}
		}
		w := C.ig_weights{
			emb_norm: (*C.float)(f32(m.EmbNorm.W)), final_norm: (*C.float)(f32(m.FinalNorm.W)),
			attn_norm: &ptrs[0][0], wqkv: &ptrs[1][0], wo: &ptrs[2][0],
			mlp_norm: &ptrs[3][0], wi: &ptrs[4][0], wo_mlp: &ptrs[5][0],
		}
		if m.Emb.W != nil { // a float32 table; an on-demand one is uploaded as stored below
			w.tok_embeddings = (*C.float)(f32(m.Emb.W))
		}
		if C.ig_model_create_multi(&cfg, &w, &devs[0], C.int32_t(len(devs)), &h) != C.IG_OK {
			return nil, fmt.Errorf("modernbert: gpu: %v", lastError())
		}
	}
	if m.Emb.W == nil {
		if err := m.setEmbeddingsGPU(h, &pin); err != nil {
			C.ig_model_destroy(h)
			return nil, err
		}
	}
	if !m.int8 {
		C.ig_model_set_int8(h, 0)
	}
	return h, nil
}

// setEmbeddingsGPU uploads the on-demand table (SetEmbeddingTable,
// infer.go:20-25) in its stored format; the float32 table is never built.
func (m *Model) setEmbeddingsGPU(h *C.ig_model, pin *runtime.Pinner) error {
	st, ok := m.embTable.(StoredTable)
	if !ok {
		// A table without stored arrays: materialize it (EmbeddingMatrix).
		emb := m.EmbeddingMatrix()
		pin.Pin(&emb[0])
		t := C.ig_embedding_table{format: C.IG_EMB_F32, f32: (*C.float)(unsafe.Pointer(&emb[0]))}
		if C.ig_model_set_embeddings(h, &t) != C.IG_OK {
			return lastError()
		}
		return nil
	}
	bf16, ids, rows, i8, scale := st.Stored()
	var t C.ig_embedding_table
	if i8 != nil {
		pin.Pin(&i8[0])
		pin.Pin(&scale[0])
		t.format = C.IG_EMB_INT8
		t.i8 = (*C.int8_t)(unsafe.Pointer(&i8[0]))
		t.scale = (*C.float)(unsafe.Pointer(&scale[0]))
	} else {
		pin.Pin(&bf16[0])
		t.format = C.IG_EMB_BF16
		t.bf16 = (*C.uint16_t)(unsafe.Pointer(&bf16[0]))
		t.n_exact = C.int32_t(len(ids))
		if len(ids) > 0 {
			pin.Pin(&ids[0])
			pin.Pin(&rows[0])
			t.exact_ids = (*C.int32_t)(unsafe.Pointer(&ids[0]))
			t.exact_rows = (*C.float)(unsafe.Pointer(&rows[0]))
		}
	}
	if C.ig_model_set_embeddings(h, &t) != C.IG_OK {
		return lastError()
	}
	return nil
}

// setInt8GPU follows SetInt8 (infer.go:119-135) on the device copy: off runs
// the reference's float32 path there.
func (m *Model) setInt8GPU(on bool) {
	g := m.gpuState()
	g.mu.Lock()
	defer g.mu.Unlock()
	if g.h != nil {
		v := C.int32_t(0)
		if on {
			v = 1
		}
		C.ig_model_set_int8(g.h, v)
	}
}

// runGPU is run (infer.go:304-430) on the device: the same sequences and
// offsets, the final states handed to done.
func (m *Model) runGPU(seqs [][]int32, done func(xn []float32, offs []int)) error {
	h, err := m.gpu()
	if err != nil {
		return err
	}
	offs := make([]int64, len(seqs)+1)
	for i, s := range seqs {
		offs[i+1] = offs[i] + int64(len(s))
	}
	N := int(offs[len(seqs)])
	io := make([]int, len(offs))
	for i, o := range offs {
		io[i] = int(o)
	}
	if N == 0 {
		done(nil, io)
		return nil
	}
	ids := make([]int32, 0, N)
	for _, s := range seqs {
		ids = append(ids, s...)
	}
	xn := make([]float32, N*m.Cfg.Hidden)
	rc := C.ig_encode(h, (*C.int32_t)(unsafe.Pointer(&ids[0])), (*C.int64_t)(unsafe.Pointer(&offs[0])),
		C.int32_t(len(seqs)), C.IG_MODE_TOKENS, (*C.float)(unsafe.Pointer(&xn[0])), C.size_t(len(xn)))
	switch rc {
	case C.IG_OK:
	case C.IG_ERR_OUT_OF_VOCAB: // the wording of infer.go:310-312
		return lastError()
	default:
		return fmt.Errorf("modernbert: gpu: %v", lastError())
	}
	done(xn, io)
	return nil
}

// encodeSeqsGPU is EncodeSeqs (infer.go:261-289) with the pooling on the
// device (the same float64 token-order mean, or the first token): only
// [len(seqs)][Hidden] comes back.
func (m *Model) encodeSeqsGPU(seqs [][]int32) ([]float32, error) {
	h, err := m.gpu()
	if err != nil {
		return nil, err
	}
	offs := make([]int64, len(seqs)+1)
	for i, s := range seqs {
		offs[i+1] = offs[i] + int64(len(s))
	}
	out := make([]float32, len(seqs)*m.Cfg.Hidden)
	N := int(offs[len(seqs)])
	if len(seqs) == 0 {
		return out, nil
	}
	ids := make([]int32, 0, N+1)
	for _, s := range seqs {
		ids = append(ids, s...)
	}
	ids = append(ids, 0) // a valid address when every sequence is empty
	rc := C.ig_encode(h, (*C.int32_t)(unsafe.Pointer(&ids[0])), (*C.int64_t)(unsafe.Pointer(&offs[0])),
		C.int32_t(len(seqs)), C.IG_MODE_POOLED, (*C.float)(unsafe.Pointer(&out[0])), C.size_t(len(out)))
	switch rc {
	case C.IG_OK:
		return out, nil
	case C.IG_ERR_OUT_OF_VOCAB:
		return nil, lastError()
	default:
		return nil, fmt.Errorf("modernbert: gpu: %v", lastError())
	}
}
