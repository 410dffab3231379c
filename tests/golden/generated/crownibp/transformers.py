import gc
import json
import os
import torch
import operator
from constraintflow.lib.globals import device_mode
from constraintflow.lib.polyexp import PolyExpSparse
from constraintflow.lib.symexp import *
from constraintflow.gbcsr.sparse_tensor import SparseTensor
from constraintflow.lib.llist import Llist
from constraintflow.gbcsr.tensor_ops import *
class crownibp:
	def Affine(self, abs_elem, prev, curr, poly_size, curr_size, prev_size, input_size, batch_size, layer_index = None):
		var_18 = any(binary(curr.get_metadata('last_layer', batch_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), SparseTensor([], [], 0, torch.tensor([]), dense_const=1, type= type(1)).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([1, curr_size])), operator.eq, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
		cse_var_24 = repeat(curr.get_metadata('bias', batch_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), torch.tensor([batch_size, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_25 = prev.dot(curr.get_metadata('weight', batch_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), abs_elem.get_poly_size(), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1, mats_input = 'rhs')
		cse_var_52 = binary(cse_var_25.get_const(), cse_var_24, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_71 = cse_var_25.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_45 = PolyExpSparse(abs_elem.network, cse_var_71 , cse_var_52)
		if(var_18):
			if dummy_mode:
				save_capture("jit_branch/branch_" + str(layer_index) + "_0.json", {"taken": "then"})
			cse_var_113 = binary(get_dims(cse_var_71, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), 1, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			vertices_stop1 = False
			cse_var_14 = SparseTensor([], [], 0, torch.tensor([]), dense_const=0.0, type= type(0.0)).unsqueeze(0).unsqueeze(1).unsqueeze(2).repeat(torch.tensor([batch_size, curr_size, poly_size]))
			cse_var_116 = Llist(abs_elem.network, [1]*(cse_var_113), None, None,torch.nonzero(abs_elem.d['llist']).flatten().tolist()).get_metadata('layer', batch_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
			cse_var_115 = Llist(abs_elem.network, [1]*(cse_var_113), None, None,torch.nonzero(abs_elem.d['llist']).flatten().tolist())
			cse_var_117 = abs_elem.get_elem('L', cse_var_115, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
			cse_var_118 = abs_elem.get_elem('U', cse_var_115, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
			cse_var_120 = cse_var_118.get_const()
			cse_var_119 = cse_var_118.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
			cse_var_122 = cse_var_117.get_const()
			cse_var_121 = cse_var_117.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
			phi_trav_exp1_2_1 = cse_var_45
			while_iteration = -1
			while(True):
				while_iteration += 1
				cse_var_28 = phi_trav_exp1_2_1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
				vertices1_2_1 = binary(cse_var_28, cse_var_14, operator.ne, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				vertices_stop_default1 = get_default_stop([batch_size, curr_size, poly_size], abs_elem, batch_size, curr_size, poly_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
				vertices_stop_temp1 = binary(SparseTensor([], [], 0, torch.tensor([]), dense_const=vertices_stop1, type= type(vertices_stop1)).unsqueeze(0).unsqueeze(1).unsqueeze(2).repeat(torch.tensor([batch_size, curr_size, poly_size])), vertices_stop_default1, operator.or_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				vertices1_2_2 = binary(vertices1_2_1, unary(vertices_stop_temp1, operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), operator.and_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				if(unary(any(vertices1_2_2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)):
					break
				priority_vertices1 = get_max_priority(cse_var_116, vertices1_2_2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
				vertices_final_stop1 = binary(vertices_stop_temp1, repeat(unary(priority_vertices1, operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), torch.tensor([batch_size, curr_size, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.or_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				polyexp_stop1 = filter_trav_exp_stop(phi_trav_exp1_2_1, vertices_final_stop1, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
				polyexp_not_stop1 = filter_trav_exp_not_stop(phi_trav_exp1_2_1, vertices_final_stop1, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
				cse_var_107 = polyexp_not_stop1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
				cse_var_104 = (cse_var_107).unsqueeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_99 = clamp(cse_var_107, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_101 = clamp(cse_var_107, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_95 = clamp(cse_var_104, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_97 = clamp(cse_var_104, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_63 = binary(inner_prod(cse_var_101, (cse_var_122).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod(cse_var_99, (cse_var_120).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_64 = binary(inner_prod((cse_var_97).squeeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (cse_var_121).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod((cse_var_95).squeeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (cse_var_119).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_62 = binary(cse_var_63, polyexp_not_stop1.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				trav_exp1_5_3 = PolyExpSparse(abs_elem.network, binary(cse_var_64, polyexp_stop1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1) , binary(cse_var_62, polyexp_stop1.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
				phi_trav_exp1_2_1 = trav_exp1_5_3
			if dummy_mode:
				json_obj = {"num_iterations": while_iteration}
				save_capture("jit_while/while_iterations_layer_" + str(layer_index) + "_while_" + str(-1) + ".json", json_obj)
			cse_var_26 = Llist(abs_elem.network, [1]*(phi_trav_exp1_2_1.mat.dims-1), None, None,torch.nonzero(abs_elem.d['llist']).flatten().tolist())
			cse_var_108 = phi_trav_exp1_2_1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
			l_new_3_0 = binary(binary(inner_prod(clamp(cse_var_108, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (abs_elem.get_elem('l', cse_var_26, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod(clamp(cse_var_108, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (abs_elem.get_elem('u', cse_var_26, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), phi_trav_exp1_2_1.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			vertices_stop2 = False
			phi_trav_exp2_6_1 = cse_var_45
			while_iteration = -1
			while(True):
				while_iteration += 1
				cse_var_15 = phi_trav_exp2_6_1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
				vertices2_6_1 = binary(cse_var_15, cse_var_14, operator.ne, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				vertices_stop_default2 = get_default_stop([batch_size, curr_size, poly_size], abs_elem, batch_size, curr_size, poly_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
				vertices_stop_temp2 = binary(SparseTensor([], [], 0, torch.tensor([]), dense_const=vertices_stop2, type= type(vertices_stop2)).unsqueeze(0).unsqueeze(1).unsqueeze(2).repeat(torch.tensor([batch_size, curr_size, poly_size])), vertices_stop_default2, operator.or_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				vertices2_6_2 = binary(vertices2_6_1, unary(vertices_stop_temp2, operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), operator.and_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				if(unary(any(vertices2_6_2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)):
					break
				priority_vertices2 = get_max_priority(cse_var_116, vertices2_6_2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
				vertices_final_stop2 = binary(vertices_stop_temp2, repeat(unary(priority_vertices2, operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), torch.tensor([batch_size, curr_size, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.or_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				polyexp_stop2 = filter_trav_exp_stop(phi_trav_exp2_6_1, vertices_final_stop2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
				polyexp_not_stop2 = filter_trav_exp_not_stop(phi_trav_exp2_6_1, vertices_final_stop2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
				cse_var_92 = polyexp_not_stop2.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
				cse_var_89 = (cse_var_92).unsqueeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_84 = clamp(cse_var_92, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_86 = clamp(cse_var_92, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_80 = clamp(cse_var_89, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_82 = clamp(cse_var_89, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_54 = binary(inner_prod(cse_var_86, (cse_var_120).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod(cse_var_84, (cse_var_122).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_55 = binary(inner_prod((cse_var_82).squeeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (cse_var_119).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod((cse_var_80).squeeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (cse_var_121).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_53 = binary(cse_var_54, polyexp_not_stop2.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				trav_exp2_9_3 = PolyExpSparse(abs_elem.network, binary(cse_var_55, polyexp_stop2.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1) , binary(cse_var_53, polyexp_stop2.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
				phi_trav_exp2_6_1 = trav_exp2_9_3
			if dummy_mode:
				json_obj = {"num_iterations": while_iteration}
				save_capture("jit_while/while_iterations_layer_" + str(layer_index) + "_while_" + str(-1) + ".json", json_obj)
			cse_var_12 = Llist(abs_elem.network, [1]*(phi_trav_exp2_6_1.mat.dims-1), None, None,torch.nonzero(abs_elem.d['llist']).flatten().tolist())
			cse_var_93 = phi_trav_exp2_6_1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
			u_new_7_0 = binary(binary(inner_prod(clamp(cse_var_93, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (abs_elem.get_elem('u', cse_var_12, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod(clamp(cse_var_93, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (abs_elem.get_elem('l', cse_var_12, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), phi_trav_exp2_6_1.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			return l_new_3_0, u_new_7_0, cse_var_45, cse_var_45, 
		else:
			if dummy_mode:
				save_capture("jit_branch/branch_" + str(layer_index) + "_0.json", {"taken": "else"})
			cse_var_51 = Llist(abs_elem.network, [1]*(cse_var_45.mat.dims-1), None, None,torch.nonzero(abs_elem.d['llist']).flatten().tolist())
			cse_var_50 = cse_var_45.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
			cse_var_77 = clamp(cse_var_50, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_78 = clamp(cse_var_50, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_111 = (abs_elem.get_elem('l', cse_var_51, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_112 = (abs_elem.get_elem('u', cse_var_51, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			l_new_10_1 = binary(binary(inner_prod(cse_var_78, cse_var_111, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod(cse_var_77, cse_var_112, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_52, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			u_new_10_1 = binary(binary(inner_prod(cse_var_78, cse_var_112, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod(cse_var_77, cse_var_111, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_52, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			return l_new_10_1, u_new_10_1, cse_var_45, cse_var_45, 
	
	def Relu(self, abs_elem, prev, curr, poly_size, curr_size, prev_size, input_size, batch_size, layer_index = None):
		cse_var_42 = abs_elem.get_elem('l', prev, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_43 = SparseTensor([], [], 0, torch.tensor([]), dense_const=0.0, type= type(0.0)).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size]))
		cse_var_47 = binary(cse_var_42, cse_var_43, operator.ge, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		rewrite_new_0 = convert_to_float(cse_var_47)
		cse_var_110 = SparseTensor([], [], 0, torch.tensor([]), dense_const=1.0, type= type(1.0)).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size]))
		l_new = binary(binary(rewrite_new_0, cse_var_42, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), binary(binary(cse_var_110, rewrite_new_0, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_43, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_41 = abs_elem.get_elem('u', prev, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		rewrite_new_1 = convert_to_float(binary(cse_var_41, cse_var_43, operator.ge, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
		u_new = binary(binary(rewrite_new_1, cse_var_41, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), binary(binary(cse_var_110, rewrite_new_1, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_43, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_39 = prev.convert_to_poly(abs_elem)
		cse_var_48 = repeat(cse_var_39.get_const(), torch.tensor([batch_size, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_49 = repeat(cse_var_39.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), torch.tensor([batch_size, 1, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_38 = PolyExpSparse(abs_elem.network, 0.0, 0.0)
		cse_var_40 = binary(binary(cse_var_42, cse_var_41, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_43, operator.ge, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_109 = convert_to_float(cse_var_40)
		rewrite_new_2 = repeat((cse_var_109).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, poly_size]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_114 = binary(cse_var_110, cse_var_109, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		L_new = PolyExpSparse(abs_elem.network, binary(binary(rewrite_new_2, cse_var_49, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), repeat((binary(cse_var_114, SparseTensor([], [], 0, torch.tensor([]), dense_const=cse_var_38.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), type= type(cse_var_38.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None))).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size])), operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, poly_size]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1) , binary(binary(cse_var_109, cse_var_48, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), binary(cse_var_114, SparseTensor([], [], 0, torch.tensor([]), dense_const=cse_var_38.get_const(), type= type(cse_var_38.get_const())).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size])), operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
		cse_var_35 = binary(cse_var_41, cse_var_42, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_37 = binary(cse_var_41, cse_var_35, operator.truediv, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_75 = binary(cse_var_37, cse_var_48, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_76 = binary(repeat((cse_var_37).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, poly_size]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_49, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_74 = binary(cse_var_75, binary(binary(cse_var_41, cse_var_42, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_35, operator.truediv, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_33 = PolyExpSparse(abs_elem.network, 0.0, cse_var_43)
		cse_var_34 = binary(cse_var_41, cse_var_43, operator.le, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_72 = where(cse_var_34, cse_var_33.get_const(), cse_var_74, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_73 = where(repeat((cse_var_34).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, poly_size]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_33.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), cse_var_76, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		U_new = PolyExpSparse(abs_elem.network, where(repeat((cse_var_47).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, poly_size]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_49, cse_var_73, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1) , where(cse_var_47, cse_var_48, cse_var_72, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
		return l_new, u_new, L_new, U_new, 
	
