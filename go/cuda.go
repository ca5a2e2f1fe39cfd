//go:build cuda

// Package llama, cuda build: the per-token path of internal/llama/infer.go
// (ForwardIntoWorkspace, ForwardTopKIntoWorkspace) and the worker pool's
// matvecs (matvec_cgo.go, workers.go) run in libl3g on the GPU.
//
// A maintainer copies this file to internal/llama/cuda.go and restricts the
// CPU implementations to the other build:
//   - infer.go and matvec_topk.go get "//go:build !cuda";
//   - matvec_cgo.go and dot_cgo.go get "//go:build cgo && !cuda".
//
// Nothing else in the package changes: Model, State and Workspace keep
// their fields, and the GPU handles live in side tables keyed by those
// pointers.  LoadModel, NewState and NewWorkspace are unchanged; the GPU
// model is uploaded on the first forward call (or explicitly with
// UploadModel), and a state's or workspace's GPU twin is created on its
// first use with the same context length.
package llama

/*
#cgo CFLAGS: -I${SRCDIR}/../../include
#cgo LDFLAGS: -L${SRCDIR}/../../llama3.go_b200 -ll3g -Wl,-rpath,${SRCDIR}/../../llama3.go_b200
#include <stdlib.h>
#include "l3g.h"
*/
import "C"

import (
	"fmt"
	"sync"
	"unsafe"
)

func l3gErr(rc C.int) error {
	if rc == C.L3G_OK {
		return nil
	}
	return fmt.Errorf("%s", C.GoString(C.l3g_last_error()))
}

var (
	gpuMu         sync.Mutex
	gpuModels     = map[*Model]*C.l3g_model{}
	gpuStates     = map[*State]*C.l3g_state{}
	gpuWorkspaces = map[*Workspace]*C.l3g_workspace{}
)

// UploadModel hands the mmapped GGUF tensors to the library once: it copies
// and repacks them into device memory and keeps no host pointer.
func (m *Model) UploadModel() error {
	gpuMu.Lock()
	defer gpuMu.Unlock()
	return m.uploadLocked()
}

func (m *Model) uploadLocked() error {
	if _, ok := gpuModels[m]; ok {
		return nil
	}
	names := make([]*C.char, 0, len(m.File.ByName))
	ts := make([]C.l3g_tensor, 0, len(m.File.ByName))
	for name, t := range m.File.ByName {
		cn := C.CString(name)
		names = append(names, cn)
		var ct C.l3g_tensor
		ct.name = cn
		ct._type = C.uint32_t(t.Info.Type)
		ct.n_dims = C.uint32_t(len(t.Info.Dims))
		for i, d := range t.Info.Dims {
			ct.dims[i] = C.uint64_t(d)
		}
		ct.data = unsafe.Pointer(&t.Data[0])
		ct.nbytes = 0 // derived from the type and dims
		ts = append(ts, ct)
	}
	defer func() {
		for _, p := range names {
			C.free(unsafe.Pointer(p))
		}
	}()
	hp := C.l3g_hparams{
		vocab_size: C.int32_t(m.HP.VocabSize), n_layers: C.int32_t(m.HP.NLayers),
		n_emb: C.int32_t(m.HP.NEmb), n_heads: C.int32_t(m.HP.NHeads),
		n_heads_kv: C.int32_t(m.HP.NHeadsKV), n_ff: C.int32_t(m.HP.NFF),
		rope_dim: C.int32_t(m.HP.RopeDim), ctx_len: C.int32_t(m.HP.CtxLen),
		rms_eps: C.float(m.HP.RmsEps), rope_base: C.float(m.HP.RopeBase),
	}
	var opt C.l3g_options
	C.l3g_options_default(&opt)
	var h *C.l3g_model
	if err := l3gErr(C.l3g_model_load(&hp, &ts[0], C.int32_t(len(ts)), &opt, &h)); err != nil {
		return err
	}
	gpuModels[m] = h
	return nil
}

// handles returns the GPU twins of (m, s, ws), creating them on first use.
func (m *Model) handles(s *State, ws *Workspace) (*C.l3g_model, *C.l3g_state, *C.l3g_workspace, error) {
	if ws == nil {
		return nil, nil, nil, fmt.Errorf("workspace is nil")
	}
	gpuMu.Lock()
	defer gpuMu.Unlock()
	if err := m.uploadLocked(); err != nil {
		return nil, nil, nil, err
	}
	mh := gpuModels[m]
	sh, ok := gpuStates[s]
	if !ok {
		if err := l3gErr(C.l3g_state_new(mh, C.int32_t(s.KV.CtxLen), &sh)); err != nil {
			return nil, nil, nil, err
		}
		gpuStates[s] = sh
	}
	if err := l3gErr(C.l3g_state_set_pos(sh, C.int32_t(s.Pos))); err != nil {
		return nil, nil, nil, err // a caller that rewinds s.Pos (main.go:120-122) rewinds the GPU state
	}
	wh, ok := gpuWorkspaces[ws]
	if !ok {
		if err := l3gErr(C.l3g_workspace_new(mh, C.int32_t(ws.CtxLen), C.int32_t(cap(ws.TopKBuf)), &wh)); err != nil {
			return nil, nil, nil, err
		}
		gpuWorkspaces[ws] = wh
	}
	return mh, sh, wh, nil
}

// ForwardIntoWorkspace replaces infer.go:21-267: one token through every
// layer; logitsOut nil skips the logits (prefill, infer.go:250).
func (m *Model) ForwardIntoWorkspace(s *State, token int32, logitsOut []float32, ws *Workspace) error {
	if logitsOut != nil && len(logitsOut) != m.HP.VocabSize {
		return fmt.Errorf("logitsOut len=%d, want %d", len(logitsOut), m.HP.VocabSize)
	}
	mh, sh, wh, err := m.handles(s, ws)
	if err != nil {
		return err
	}
	var out *C.float
	if logitsOut != nil {
		out = (*C.float)(unsafe.Pointer(&logitsOut[0]))
	}
	if err := l3gErr(C.l3g_forward(mh, sh, wh, C.int32_t(token), out)); err != nil {
		return err
	}
	s.Pos++ // mirrors the device state's position (infer.go:265)
	return nil
}

// ForwardTopKIntoWorkspace replaces infer.go:269-511.  TopKItem{int32,
// float32} has the C layout of l3g_topk_item.  Items come back sorted by
// descending logit; SampleTopK accepts either order.
func (m *Model) ForwardTopKIntoWorkspace(s *State, token int32, topK int, ws *Workspace) ([]TopKItem, error) {
	if topK <= 0 {
		topK = 40
	}
	mh, sh, wh, err := m.handles(s, ws)
	if err != nil {
		return nil, err
	}
	items := make([]TopKItem, topK)
	var n C.int32_t
	rc := C.l3g_forward_topk(mh, sh, wh, C.int32_t(token), C.int32_t(topK),
		(*C.l3g_topk_item)(unsafe.Pointer(&items[0])), &n)
	if err := l3gErr(rc); err != nil {
		return nil, err
	}
	s.Pos++
	return items[:n], nil
}

// UseFastExpTopK makes ws's top-K and sampled calls weight attention
// positions with the reference top-K path's fastExp (infer.go:404,520-525),
// so they return that path's items; call it once after NewWorkspace.
func (m *Model) UseFastExpTopK(s *State, ws *Workspace) error {
	_, _, wh, err := m.handles(s, ws)
	if err != nil {
		return err
	}
	return l3gErr(C.l3g_workspace_set_topk_fast_exp(wh, 1))
}

// DecodeSample runs a whole reply on the device: sampling (SampleTopK,
// sampling.go:103-143, with Philox draws keyed by seed) and the chat loop's
// stop rule (main.go:146-150).  It returns the sampled ids through the
// first stop id.
func (m *Model) DecodeSample(s *State, ws *Workspace, next int32, maxTokens, topK int,
	temp float32, seed uint64, stops []int32) ([]int32, error) {
	mh, sh, wh, err := m.handles(s, ws)
	if err != nil {
		return nil, err
	}
	out := make([]int32, maxTokens)
	var n C.int32_t
	var stopPtr *C.int32_t
	if len(stops) > 0 {
		stopPtr = (*C.int32_t)(unsafe.Pointer(&stops[0]))
	}
	rc := C.l3g_decode_sample(mh, sh, wh, C.int32_t(next), C.int32_t(maxTokens),
		C.int32_t(topK), C.float(temp), C.uint64_t(seed), stopPtr, C.int32_t(len(stops)),
		(*C.int32_t)(unsafe.Pointer(&out[0])), &n, nil)
	if err := l3gErr(rc); err != nil {
		return nil, err
	}
	var pos C.int32_t
	if err := l3gErr(C.l3g_state_pos(sh, &pos)); err != nil {
		return nil, err
	}
	s.Pos = int(pos)
	return out[:n], nil
}

// Snapshot and Restore keep a session's KV prefix in host memory, e.g. for
// the chat loop's /reset (main.go:120-122) without re-ingesting the system
// prompt.
func (m *Model) Snapshot(s *State, ws *Workspace) ([]byte, error) {
	_, sh, _, err := m.handles(s, ws)
	if err != nil {
		return nil, err
	}
	var n C.uint64_t
	if err := l3gErr(C.l3g_state_snapshot_bytes(sh, &n)); err != nil {
		return nil, err
	}
	buf := make([]byte, int(n))
	if err := l3gErr(C.l3g_state_snapshot(sh, unsafe.Pointer(&buf[0]), n)); err != nil {
		return nil, err
	}
	return buf, nil
}

func (m *Model) Restore(s *State, ws *Workspace, snap []byte) error {
	_, sh, _, err := m.handles(s, ws)
	if err != nil {
		return err
	}
	if err := l3gErr(C.l3g_state_restore(sh, unsafe.Pointer(&snap[0]), C.uint64_t(len(snap)))); err != nil {
		return err
	}
	var pos C.int32_t
	if err := l3gErr(C.l3g_state_pos(sh, &pos)); err != nil {
		return err
	}
	s.Pos = int(pos)
	return nil
}

// Batch steps many sessions together (no counterpart in the reference's
// chat loop, which serves one session).
type Batch struct{ h *C.l3g_batch }

func (m *Model) NewBatch(maxSeqs int) (*Batch, error) {
	gpuMu.Lock()
	defer gpuMu.Unlock()
	if err := m.uploadLocked(); err != nil {
		return nil, err
	}
	var h *C.l3g_batch
	if err := l3gErr(C.l3g_batch_new(gpuModels[m], C.int32_t(maxSeqs), &h)); err != nil {
		return nil, err
	}
	return &Batch{h: h}, nil
}

// Step advances every session by one token: per session the top-K forward
// and SampleTopK on the device; next receives the sampled ids.
func (m *Model) Step(b *Batch, states []*State, ws *Workspace, tokens []int32, topK int,
	temp float32, seeds []uint64) ([]int32, error) {
	hs := make([]*C.l3g_state, len(states))
	for i, s := range states {
		_, sh, _, err := m.handles(s, ws)
		if err != nil {
			return nil, err
		}
		hs[i] = sh
	}
	next := make([]int32, len(states))
	rc := C.l3g_batch_step(b.h, (**C.l3g_state)(unsafe.Pointer(&hs[0])), C.int32_t(len(hs)),
		(*C.int32_t)(unsafe.Pointer(&tokens[0])), C.int32_t(topK), C.float(temp),
		(*C.uint64_t)(unsafe.Pointer(&seeds[0])), (*C.int32_t)(unsafe.Pointer(&next[0])), nil)
	if err := l3gErr(rc); err != nil {
		return nil, err
	}
	for _, s := range states {
		s.Pos++
	}
	return next, nil
}

func (b *Batch) Close() {
	if b.h != nil {
		C.l3g_batch_free(b.h)
		b.h = nil
	}
}

// Close releases the GPU twins (a process holds one model): workspaces
// first (their step graphs hold the model's communicator), then states,
// then the model.
func (m *Model) Close() {
	gpuMu.Lock()
	defer gpuMu.Unlock()
	for ws, h := range gpuWorkspaces {
		C.l3g_workspace_free(h)
		delete(gpuWorkspaces, ws)
	}
	for s, h := range gpuStates {
		C.l3g_state_free(h)
		delete(gpuStates, s)
	}
	if h, ok := gpuModels[m]; ok {
		C.l3g_model_free(h)
		delete(gpuModels, m)
	}
}
